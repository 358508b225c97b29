"""The decoder around the path on the GPU: its kernels (embedding lookup from
the 4-bit table, RMSNorm, RoPE) against the oracle / fp32 math, the attention
half of a block against an fp32 restatement, and the decoder's three decode
forms (prefill, eager windows, the CUDA-graph step) against each other."""
from __future__ import annotations

import math

import numpy as np
import pytest

from conftest import rel_l2

pytestmark = pytest.mark.gpu


def _np(t):
    from b2q.synth import to_numpy_bits

    return to_numpy_bits(t)


def _bf(a):
    from oracle.oracle import bf16_to_f32

    return bf16_to_f32(a)


def _tiny(**kw):
    from b2q.model import DecoderConfig

    c = dict(n_layers=2, hidden=1024, n_heads=8, n_kv_heads=2, head_dim=128, n_experts=16, top_k=4,
             expert_ffn=512, vocab=4096, max_seq=64, mtp=True)
    c.update(kw)
    return DecoderConfig(**c)


def test_embed_gather_is_the_dequantized_rows(cuda, b2q_mod, oracle):
    import torch

    from b2q.model import Decoder

    dec = Decoder(_tiny(n_layers=1, mtp=False), seed=3)
    ids = torch.tensor([0, 4095, 17, 17, 2048], dtype=torch.int32, device="cuda")
    got = _np(dec.embed(ids))
    rows = ids.cpu().numpy()
    ref = oracle.dequantize(_np(dec.embed_w)[rows], _np(dec.embed_s)[rows], _np(dec.embed_b)[rows], 64,
                            variant="metal")
    assert np.array_equal(got, ref)
    assert dec.status() == 0
    bad = torch.tensor([5, 4096], dtype=torch.int32, device="cuda")
    out = _np(dec.embed(bad))
    assert dec.status() == b2q_mod._lib.B2Q_EINVAL and not out[1].any()


def test_rms_norm_and_rope(cuda, b2q_mod):
    import torch

    from b2q import synth
    from b2q._lib import check, lib
    from b2q.model import rms_norm

    x = synth.activations((5, 1024), seed=40) * 3
    w = (1.0 + 0.1 * synth.activations((1024,), seed=41)).to(torch.bfloat16)
    got = _bf(_np(rms_norm(x, w, 1e-6)))
    xf, wf = _bf(_np(x)).astype(np.float64), _bf(_np(w)).astype(np.float64)
    ref = xf / np.sqrt((xf ** 2).mean(-1, keepdims=True) + 1e-6) * wf
    assert np.abs(got - ref).max() <= np.abs(ref).max() * 2 ** -7
    assert rel_l2(got, ref) < 3e-3
    # rope over [T, heads, d] at given positions, theta 1e6
    T, heads, d = 3, 4, 128
    q = synth.activations((T, heads, d), seed=42)
    pos = torch.tensor([0, 7, 1000], dtype=torch.int32, device="cuda")
    qr = q.clone()
    check(lib().b2q_rope(qr.data_ptr(), T, heads, d, pos.data_ptr(), 0, 1e6, torch.cuda.current_stream().cuda_stream))
    a = _bf(_np(q)).astype(np.float64)
    half = d // 2
    inv = 1e6 ** (-np.arange(half) / half)
    ang = pos.cpu().numpy()[:, None, None].astype(np.float64) * inv[None, None, :]
    x1, x2 = a[..., :half], a[..., half:]
    ref = np.concatenate([x1 * np.cos(ang) - x2 * np.sin(ang), x1 * np.sin(ang) + x2 * np.cos(ang)], -1)
    assert rel_l2(_bf(_np(qr)), ref) < 5e-3
    assert np.array_equal(_np(qr)[0], _bf16_round(ref[0]))


def _bf16_round(a):
    from oracle.oracle import f32_to_bf16

    return f32_to_bf16(np.asarray(a, np.float32))


def _attention_half_reference(blk, h, pos0, k_hist, v_hist):
    """fp32 restatement of h + o(attention(rms_norm(h))) with dequantized weights,
    rounding to bf16 where the device path stores bf16."""
    import torch

    from b2q import ops

    cfg = blk.cfg
    nq, nk, hd = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
    f = lambda t: torch.from_numpy(_bf(_np(t)).astype(np.float32))  # noqa: E731
    rb = lambda t: t.to(torch.bfloat16).float()  # noqa: E731
    wqkv = f(ops.dequantize(blk.qkv.weight, blk.qkv.scales, blk.qkv.biases))
    wo = f(ops.dequantize(blk.o.weight, blk.o.scales, blk.o.biases))
    x = f(h)
    T = x.shape[0]
    a = rb(x * torch.rsqrt((x * x).mean(-1, keepdim=True) + cfg.rms_eps) * f(blk.attn_norm))
    qkv = rb(a @ wqkv.T)
    q, k, v = qkv[:, :nq * hd], qkv[:, nq * hd:(nq + nk) * hd], qkv[:, (nq + nk) * hd:]
    half = hd // 2
    pos = torch.arange(pos0, pos0 + T, dtype=torch.float64)
    inv = torch.tensor(cfg.rope_theta, dtype=torch.float64) ** (-torch.arange(half, dtype=torch.float64) / half)
    ang = (pos[:, None] * inv[None, :])
    cs, sn = torch.cos(ang).float()[:, None, :], torch.sin(ang).float()[:, None, :]

    def rope(t, heads):
        t = t.view(T, heads, hd)
        x1, x2 = t[..., :half], t[..., half:]
        return rb(torch.cat([x1 * cs - x2 * sn, x1 * sn + x2 * cs], -1))

    q, k = rope(q, nq), rope(k, nk)
    K = torch.cat([k_hist, k]) if k_hist is not None else k
    V = torch.cat([v_hist, v.view(T, nk, hd)]) if v_hist is not None else v.view(T, nk, hd)
    g = nq // nk
    out = torch.zeros(T, nq, hd)
    for t in range(T):
        for hq in range(nq):
            kv = hq // g
            s = (K[:pos0 + t + 1, kv] @ q[t, hq]) / math.sqrt(hd)
            p = torch.softmax(s, 0)
            out[t, hq] = p @ V[:pos0 + t + 1, kv]
    o = rb(rb(out.view(T, nq * hd)) @ wo.T)
    return rb(x + o), K, V


def test_attention_half_against_fp32(cuda, b2q_mod):
    """Prefill of 12 rows, then a 2-row window at position 12 on the filled cache."""
    import torch

    from b2q import synth
    from b2q.model import Block, rms_norm

    cfg = _tiny()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    ws = torch.zeros(b2q_mod.lib().b2q_attn_decode_workspace_size(8, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim,
                                                                   cfg.max_seq), dtype=torch.uint8, device="cuda")
    blk = Block(cfg, torch.device("cuda"), 50, status, ws)
    h = synth.activations((12, cfg.hidden), seed=51)
    pos = torch.arange(12, dtype=torch.int32, device="cuda")
    got = h + blk.o(blk.attention(rms_norm(h, blk.attn_norm, cfg.rms_eps), pos, 0))
    ref, K, V = _attention_half_reference(blk, h, 0, None, None)
    assert rel_l2(_bf(_np(got)), ref.numpy()) < 1e-2
    h2 = synth.activations((2, cfg.hidden), seed=52)
    pos2 = torch.arange(12, 14, dtype=torch.int32, device="cuda")
    got2 = h2 + blk.o(blk.attention(rms_norm(h2, blk.attn_norm, cfg.rms_eps), pos2))
    ref2, _, _ = _attention_half_reference(blk, h2, 12, K, V)
    assert rel_l2(_bf(_np(got2)), ref2.numpy()) < 1e-2
    assert int(status.item()) == 0


def test_decoder_decode_forms_agree(cuda, b2q_mod):
    """The logits of position 9 from (a) a 10-token prefill, (b) a 9-token prefill
    then a one-row window, (c) the CUDA-graph step; and greedy generation with and
    without the draft head starts from the same token."""
    import torch

    from b2q.model import Decoder

    cfg = _tiny()
    dec = Decoder(cfg, seed=7)
    g = torch.Generator(device="cuda")
    g.manual_seed(8)
    ids = torch.randint(0, cfg.vocab, (10,), generator=g, device="cuda", dtype=torch.int32)
    _, la = dec.forward(ids, 0)
    la = _bf(_np(la)).reshape(-1)
    _, _ = dec.forward(ids[:9], 0)
    hb = dec._window(ids[9:10], 9)
    lb = _bf(_np(dec.logits(hb))).reshape(-1)
    assert rel_l2(lb, la) < 2e-2
    replay, tok, pos, lg = dec.decode_graph()
    _, _ = dec.forward(ids[:9], 0)
    tok.fill_(int(ids[9]))
    pos.fill_(9)
    replay()
    torch.cuda.synchronize()
    lc = _bf(_np(lg)).reshape(-1)
    assert rel_l2(lc, la) < 2e-2
    assert int(pos.item()) == 10 and lc[int(tok.item())] == lc.max()
    # a second replay continues from the graph's own token / position
    replay()
    torch.cuda.synchronize()
    assert int(pos.item()) == 11
    assert dec.status() == 0
    t0, _ = dec.generate(ids, 4)
    t1, acc = dec.generate(ids, 5, use_mtp=True)
    assert len(t0) == 4 and len(t1) == 5 and t0[0] == t1[0] and 0 <= acc <= 2


def test_graph_token_stream_matches_eager_windows(cuda, b2q_mod):
    """Sixteen greedy tokens from the CUDA-graph step against the eager one-row
    windows, on a model whose output varies: with the tied table a random model
    keeps predicting its input token, so the lm_head rows are a rotation of the
    embedding rows (the prediction moves to another token every step)."""
    import torch

    from b2q.model import Decoder
    from b2q.nn import QuantizedLinear

    cfg = _tiny()
    dec = Decoder(cfg, seed=11)
    perm = torch.randperm(cfg.vocab, generator=torch.Generator().manual_seed(12)).cuda()
    rows = lambda t: t.view(torch.int16 if t.element_size() == 2 else torch.int32)[perm].contiguous().view(t.dtype)
    dec.lm_head = QuantizedLinear(rows(dec.embed_w), rows(dec.embed_s), rows(dec.embed_b), cfg.group_size, 4)
    g = torch.Generator(device="cuda")
    g.manual_seed(13)
    ids = torch.randint(0, cfg.vocab, (8,), generator=g, device="cuda", dtype=torch.int32)
    n = 16
    # graph: prefill, then replays that read and write token / position on the device
    replay, tok, pos, _ = dec.decode_graph()
    _, lg = dec.forward(ids, 0)
    graph = [int(lg.argmax(-1).item())]
    tok.fill_(graph[0])
    pos.fill_(8)
    for _ in range(n - 1):
        replay()
        graph.append(int(tok.item()))
    assert dec.status() == 0
    assert len(set(graph)) > 1, graph
    # eager one-row windows fed the graph's tokens (the KV rows are rewritten in
    # the same order): every step's argmax is the graph's next token, up to
    # near-ties of the two logits
    dec.forward(ids, 0)
    for i in range(n - 1):
        hw = dec._window(torch.tensor([graph[i]], dtype=torch.int32, device="cuda"), 8 + i)
        le = _bf(_np(dec.logits(hw))).reshape(-1)
        e = int(le.argmax())
        if e != graph[i + 1]:
            assert le[e] - le[graph[i + 1]] <= 1e-2 * np.abs(le).max(), (i, e, graph[i + 1])


def test_fused_norm_rope_kv_and_gqa_decode(cuda, b2q_mod):
    """add_rms_norm = bf16 add then the norm; rope_kv = rope in place + cache rows;
    gqa_decode over 3 key chunks (positions 5, 130, 299) against fp32 softmax attention."""
    import torch

    from b2q import synth
    from b2q._lib import check, lib
    from b2q.model import add_rms_norm, rms_norm

    st = torch.cuda.current_stream().cuda_stream
    h = synth.activations((3, 1024), seed=60) * 4
    d = synth.activations((3, 1024), seed=61)
    w = (1.0 + 0.1 * synth.activations((1024,), seed=62)).to(torch.bfloat16)
    h_ref = (h.float() + d.float()).to(torch.bfloat16)
    out = add_rms_norm(h, d, w, 1e-6)
    assert torch.equal(h, h_ref)  # in place, one bf16 rounding
    assert torch.equal(out, rms_norm(h_ref, w, 1e-6))

    nq, nk, hd, S = 8, 2, 128, 300
    T = 3
    qkv = synth.activations((T, (nq + 2 * nk) * hd), seed=63)
    pos = torch.tensor([5, 130, 299], dtype=torch.int32, device="cuda")
    kc = synth.activations((S, nk, hd), seed=64)
    vc = synth.activations((S, nk, hd), seed=65)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    q_ref = qkv[:, :nq * hd].clone().contiguous()
    k_ref = qkv[:, nq * hd:(nq + nk) * hd].clone().contiguous()
    check(lib().b2q_rope(q_ref.data_ptr(), T, nq, hd, pos.data_ptr(), 0, 1e6, st))
    check(lib().b2q_rope(k_ref.data_ptr(), T, nk, hd, pos.data_ptr(), 0, 1e6, st))
    x = qkv.clone()
    check(lib().b2q_rope_kv(x.data_ptr(), T, nq, nk, hd, pos.data_ptr(), 1e6, kc.data_ptr(), vc.data_ptr(), S,
                            status.data_ptr(), st))
    assert torch.equal(x[:, :nq * hd], q_ref) and torch.equal(x[:, nq * hd:(nq + nk) * hd], k_ref)
    pl = pos.long()
    assert torch.equal(kc[pl].reshape(T, -1), k_ref)
    assert torch.equal(vc[pl].reshape(T, -1), qkv[:, (nq + nk) * hd:])
    ws = torch.empty(lib().b2q_gqa_decode_workspace_size(T, nq, nk, hd, S), dtype=torch.uint8, device="cuda")
    out = torch.empty((T, nq * hd), dtype=torch.bfloat16, device="cuda")
    check(lib().b2q_gqa_decode(x.data_ptr(), (nq + 2 * nk) * hd, kc.data_ptr(), vc.data_ptr(), pos.data_ptr(),
                               out.data_ptr(), T, nq, nk, hd, S, status.data_ptr(), ws.data_ptr(), ws.numel(), st))
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    qf, kf, vf = x[:, :nq * hd].float().view(T, nq, hd), kc.float(), vc.float()
    ref = torch.empty(T, nq, hd, device="cuda")
    for t in range(T):
        p = int(pos[t])
        for j in range(nq):
            s = (kf[:p + 1, j // (nq // nk)] @ qf[t, j]) / hd ** 0.5
            ref[t, j] = torch.softmax(s, 0) @ vf[:p + 1, j // (nq // nk)]
    assert rel_l2(_bf(_np(out)), ref.view(T, -1).cpu().numpy()) < 4e-3
    # a position outside the window is recorded
    bad = torch.tensor([300], dtype=torch.int32, device="cuda")
    check(lib().b2q_gqa_decode(x.data_ptr(), (nq + 2 * nk) * hd, kc.data_ptr(), vc.data_ptr(), bad.data_ptr(),
                               out.data_ptr(), 1, nq, nk, hd, S, status.data_ptr(), ws.data_ptr(), ws.numel(), st))
    torch.cuda.synchronize()
    assert int(status.item()) == b2q_mod._lib.B2Q_EINVAL


def test_expert_parallel_decoder_one_rank(cuda, b2q_mod):
    """The expert-parallel decoder on one rank (all experts local, the EP decode and
    prefill operators with their fp32 partials) agrees with the plain decoder built
    from the same seeds, in prefill and in the CUDA-graph step."""
    import torch

    from b2q.model import Decoder

    cfg = _tiny(mtp=False)
    ref = Decoder(cfg, seed=21)
    dec = Decoder(cfg, seed=21, expert_parallel=(None, 1, 0))
    g = torch.Generator(device="cuda")
    g.manual_seed(22)
    ids = torch.randint(0, cfg.vocab, (12,), generator=g, device="cuda", dtype=torch.int32)
    _, la = ref.forward(ids, 0)
    _, lb = dec.forward(ids, 0)
    assert rel_l2(_bf(_np(lb)), _bf(_np(la))) < 2e-2
    replay, tok, pos, lg = dec.decode_graph()
    dec.forward(ids[:11], 0)
    tok.fill_(int(ids[11]))
    pos.fill_(11)
    replay()
    torch.cuda.synchronize()
    assert rel_l2(_bf(_np(lg)).reshape(-1), _bf(_np(la)).reshape(-1)) < 2e-2
    assert dec.status() == 0


@pytest.mark.parametrize("positions,hd,nk,S", [([0], 128, 4, 1280), ([63], 128, 4, 1280), ([64], 128, 4, 1280),
                                                ([1279], 128, 4, 1280), ([62, 63, 64], 128, 4, 1280),
                                                ([5, 130, 299], 128, 4, 1280), ([127, 128], 128, 4, 1280),
                                                ([513, 514], 128, 4, 1280), ([8703], 128, 4, 8704),
                                                ([1000, 1001], 128, 2, 1280),
                                                ([1279], 64, 4, 1280), ([62, 63, 64], 64, 4, 1280)])
def test_attn_decode_matches_two_kernel_path(cuda, b2q_mod, positions, hd, nk, S):
    """b2q_attn_decode (one launch) = b2q_rope_kv + b2q_gqa_decode: identical
    cache rows, outputs within rounding, and both against fp32 softmax
    attention; the window's own rows are read from q|k|v (rows 62, 63, 64 cross
    a chunk boundary). Two calls in a row on one workspace (its counters
    re-arm). The one-launch kernel multiplies bf16 probabilities by V on the
    tensor cores (normalised by the fp32 sum) where the two-kernel path keeps
    them in fp32, so the two paths are held to the bound each meets against
    fp32 attention (4e-3), not to each other's rounding."""
    import torch

    from b2q import synth
    from b2q._lib import check, lib

    st = torch.cuda.current_stream().cuda_stream
    nq = 32  # head_dim 128: the cluster kernel; 64: the chunk-partials kernel; nk 2: 16 q heads per kv head
    T = len(positions)
    qkv = synth.activations((T, (nq + 2 * nk) * hd), seed=70 + T)
    pos = torch.tensor(positions, dtype=torch.int32, device="cuda")
    kc0 = synth.activations((S, nk, hd), seed=71)
    vc0 = synth.activations((S, nk, hd), seed=72)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    # the two-kernel path
    x = qkv.clone()
    kc1, vc1 = kc0.clone(), vc0.clone()
    check(lib().b2q_rope_kv(x.data_ptr(), T, nq, nk, hd, pos.data_ptr(), 1e6, kc1.data_ptr(), vc1.data_ptr(), S,
                            status.data_ptr(), st))
    ws1 = torch.empty(lib().b2q_gqa_decode_workspace_size(T, nq, nk, hd, S), dtype=torch.uint8, device="cuda")
    ref = torch.empty((T, nq * hd), dtype=torch.bfloat16, device="cuda")
    check(lib().b2q_gqa_decode(x.data_ptr(), (nq + 2 * nk) * hd, kc1.data_ptr(), vc1.data_ptr(), pos.data_ptr(),
                               ref.data_ptr(), T, nq, nk, hd, S, status.data_ptr(), ws1.data_ptr(), ws1.numel(), st))
    # the fused path
    ws2 = torch.zeros(lib().b2q_attn_decode_workspace_size(T, nq, nk, hd, S), dtype=torch.uint8, device="cuda")
    for _ in range(2):
        kc2, vc2 = kc0.clone(), vc0.clone()
        out = torch.empty((T, nq * hd), dtype=torch.bfloat16, device="cuda")
        check(lib().b2q_attn_decode(qkv.data_ptr(), (nq + 2 * nk) * hd, pos.data_ptr(), kc2.data_ptr(),
                                    vc2.data_ptr(), out.data_ptr(), T, nq, nk, hd, 1e6, S, status.data_ptr(),
                                    ws2.data_ptr(), ws2.numel(), st))
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        assert torch.equal(kc2, kc1) and torch.equal(vc2, vc1)
        assert rel_l2(_bf(_np(out)), _bf(_np(ref))) < 4e-3
    qf, kf, vf = x[:, :nq * hd].float().view(T, nq, hd), kc1.float(), vc1.float()
    exact = torch.empty(T, nq, hd, device="cuda")
    for t in range(T):
        p = positions[t]
        for j in range(nq):
            s = (kf[:p + 1, j // (nq // nk)] @ qf[t, j]) / hd ** 0.5
            exact[t, j] = torch.softmax(s, 0) @ vf[:p + 1, j // (nq // nk)]
    assert rel_l2(_bf(_np(out)), exact.view(T, -1).cpu().numpy()) < 4e-3


@pytest.mark.parametrize("with_delta", [True, False])
def test_norm_fused_products(cuda, b2q_mod, with_delta):
    """b2q_qmv_norm / b2q_moe_decode_norm = b2q_add_rms_norm then b2q_qmm /
    b2q_moe_decode: the residual sum bit for bit, the products within rounding
    (the fused norm sums the squares in another order, so a normalised value
    can differ in its last bit); two calls in a row."""
    import torch

    from b2q import synth
    from b2q._lib import check, lib
    from b2q.model import add_rms_norm

    st = torch.cuda.current_stream().cuda_stream
    H, N, E, F, k = 4096, 5120, 32, 1536, 8
    h = synth.activations((1, H), seed=90) * 3
    delta = synth.activations((1, H), seed=91) if with_delta else None
    nw = (1.0 + 0.1 * synth.activations((H,), seed=92)).to(torch.bfloat16)
    w, s, b = synth.packed_weights((N,), H, 64, seed=93)
    h_ref = h.clone()
    a = add_rms_norm(h_ref, delta, nw, 1e-6)  # h_ref += delta in place
    y_ref = b2q_mod.quantized_matmul(a, w, s, b)
    L = synth.moe_layer(E, H, F, 64, seed=94)
    wr = synth.router_weight(E, H, seed=95)
    moe = b2q_mod.MoE(wr, L, k, 64)
    out_ref = moe(a)
    for _ in range(2):
        h_out = torch.full_like(h, 7.0)
        y = torch.empty((1, N), dtype=torch.bfloat16, device="cuda")
        check(lib().b2q_qmv_norm(h.data_ptr(), None if delta is None else delta.data_ptr(), nw.data_ptr(), 1e-6,
                                 h_out.data_ptr() if with_delta else None, w.data_ptr(), s.data_ptr(), b.data_ptr(),
                                 y.data_ptr(), N, H, 64, 4, st))
        torch.cuda.synchronize()
        if with_delta:
            assert torch.equal(h_out, h_ref)
        assert rel_l2(_bf(_np(y)), _bf(_np(y_ref))) < 2e-3
        h_out2 = torch.full_like(h, 7.0)
        out = moe.decode_norm(h, delta, nw, 1e-6, h_out2 if with_delta else None)
        torch.cuda.synchronize()
        if with_delta:
            assert torch.equal(h_out2, h_ref)
        assert rel_l2(_bf(_np(out)), _bf(_np(out_ref))) < 5e-3
