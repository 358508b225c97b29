"""Expert-parallel layers on the GPU.

One GPU: the layer computed as two expert shards (no communicator; each call
returns its fp32 partial) and summed matches the oracle layer, for decode and
prefill. Two or more GPUs: two ranks with an NCCL communicator of the library
produce the same output on both ranks, matching the single-GPU layer.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

from conftest import REL_L2, rel_l2

pytestmark = pytest.mark.gpu


def _np(t):
    from b2q.synth import to_numpy_bits

    return to_numpy_bits(t)


def _bf(a):
    from oracle.oracle import bf16_to_f32

    return bf16_to_f32(a)


def _layer(E, H, F, seed):
    from b2q import synth

    return synth.moe_layer(E, H, F, 64, seed=seed), synth.router_weight(E, H, seed=seed + 1)


@pytest.mark.parametrize("T", [1, 3, 96])
def test_two_shards_sum_to_the_layer(cuda, b2q_mod, oracle, T):
    from b2q import synth
    from b2q.ep import EPMoE, expert_range, shard_layer

    E, H, F, k = 16, 1024, 512, 4
    L, wr = _layer(E, H, F, 90)
    x = synth.activations((T, H), seed=92)
    total = None
    for r in range(2):
        lo, n = expert_range(E, 2, r)
        moe = EPMoE(wr, shard_layer(L, lo, n), E, lo, k)
        out, part = moe(x, return_partial=True)
        assert np.array_equal(_np(out), _np(part.to(__import__("torch").bfloat16)))
        total = part if total is None else total + part
    lg = b2q_mod.router_logits(x, wr)
    ridx, rw = oracle.route(_np(lg), k)
    Lnp = {kk: _np(v) for kk, v in L.items()}
    fn = oracle.moe_experts_decode if T <= 8 else oracle.moe_experts_prefill
    rows = None if T <= 8 else list(range(0, T, 7))
    ref = _bf(fn(_np(x), ridx, rw, Lnp, k, rows=rows))
    got = total.cpu().numpy()
    if rows is not None:
        got = got[rows]
    e = rel_l2(got, ref)
    assert e < REL_L2, e


@pytest.mark.parametrize("T", [1, 64])
@pytest.mark.parametrize("nshards", [3, 4, 8])
def test_config1_shards_sum_to_the_layer(cuda, b2q_mod, nshards, T):
    """The configuration-1 layer (E 128, top 8, H 4096, F 1536) as 3, 4 or 8
    expert shards of the one-token expert-parallel kernel (43/43/42, 32 or 16
    experts per shard, shards holding none of the token's experts included):
    the fp32 partials sum to the single-GPU layer, for one token (the
    single-column kernel) and a 64-token window (the tensor-core products over
    the shard's sorted rows). These are the kernels each rank runs at 2..8 GPUs,
    checked on one GPU."""
    import torch

    from b2q import synth
    from b2q.ep import EPMoE, expert_range, shard_layer

    E, H, F, k = 128, 4096, 1536, 8
    L, wr = _layer(E, H, F, 120)
    ref_moe = b2q_mod.MoE(wr, L, k, 64)
    for seed in (121, 122):
        x = synth.activations((T, H), seed=seed)
        ref = ref_moe(x)
        total = torch.zeros((T, H), dtype=torch.float32, device="cuda")
        for r in range(nshards):
            lo, n = expert_range(E, nshards, r)
            _, part = EPMoE(wr, shard_layer(L, lo, n), E, lo, k)(x, return_partial=True)
            total += part
        e = rel_l2(total.cpu().numpy(), _bf(_np(ref)))
        assert e < 5e-3, e


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, T, path):
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import sys

        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        sys.path[:0] = [root, os.path.join(root, "mlxfast-qwen38-125b-a6b-engine_b200")]
        from b2q import synth
        from b2q.ep import EPComm, EPMoE, expert_range, shard_layer

        E, H, F, k = 16, 1024, 512, 4
        L = synth.moe_layer(E, H, F, 64, device="cuda", seed=90)
        wr = synth.router_weight(E, H, device="cuda", seed=91)
        x = synth.activations((T, H), device="cuda", seed=92)
        comm = EPComm(world, rank)
        lo, n = expert_range(E, world, rank)
        out = EPMoE(wr, shard_layer(L, lo, n), E, lo, k, comm)(x)
        torch.cuda.synchronize()
        np.save(path + f".{rank}.npy", _np(out))
        comm.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("T", [1, 96])
def test_two_ranks_nccl(cuda, b2q_mod, tmp_path, T):
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    from b2q import synth

    path = str(tmp_path / "out")
    env = dict(os.environ)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    try:
        mp.start_processes(_rank, args=(2, _free_port(), T, path), nprocs=2, start_method="spawn", join=True)
    finally:
        os.environ.clear()
        os.environ.update(env)
    o0, o1 = np.load(path + ".0.npy"), np.load(path + ".1.npy")
    assert np.array_equal(o0, o1)
    E, H, F, k = 16, 1024, 512, 4
    L = synth.moe_layer(E, H, F, 64, seed=90)
    wr = synth.router_weight(E, H, seed=91)
    x = synth.activations((T, H), seed=92)
    ref = b2q_mod.moe_decode(x, wr, L, k) if T <= 8 else b2q_mod.moe_prefill(x, wr, L, k)
    assert rel_l2(_bf(o0), _bf(_np(ref))) < REL_L2


def _peer_case(E, H, F, device):
    """Three layers: two with random routers, one whose router sends every token
    to experts 0..3 (rank 0's), so the other ranks hold none of the token's
    experts (their partial is zero); tokens with positive entries."""
    import torch

    from b2q import synth

    layers = [synth.moe_layer(E, H, F, 64, device=device, seed=90 + 10 * i) for i in range(3)]
    wrs = [synth.router_weight(E, H, device=device, seed=91 + 10 * i) for i in range(2)]
    w3 = torch.full((E, H), -0.01, dtype=torch.float32, device=device)
    w3[:4] = 0.01
    wrs.append(w3.to(torch.bfloat16))
    xs = synth.activations((9, H), device=device, seed=92).abs()
    return layers, wrs, xs


def _rank_peer(rank, world, port, path):
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import sys

        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        sys.path[:0] = [root, os.path.join(root, "mlxfast-qwen38-125b-a6b-engine_b200")]
        from b2q import synth
        from b2q.ep import EPComm, EPMoE, expert_range, shard_layer

        E, H, F, k = 16, 1024, 512, 4
        layers, wrs, xs = _peer_case(E, H, F, "cuda")
        comm = EPComm(world, rank)
        lo, n = expert_range(E, world, rank)
        moes = [EPMoE(wrs[i], shard_layer(layers[i], lo, n), E, lo, k, comm) for i in range(3)]
        # nine one-token calls cycling the three layers: NCCL all-reduce, then
        # the same calls with the reduction over peer memory
        ref = [moes[i % 3](xs[i:i + 1]).clone() for i in range(9)]
        comm.enable_peer(H)
        got = [moes[i % 3](xs[i:i + 1]).clone() for i in range(9)]
        torch.cuda.synchronize()
        for i in range(3):
            st = moes[i]._ws.get("decode")
            assert int(st.view(torch.int32)[0].item()) == 0, "device-side error in the peer exchange"
        np.save(path + f".{rank}.npy", np.stack([_np(t) for t in ref + got]))
        comm.close()
    finally:
        dist.destroy_process_group()


def test_two_ranks_peer_decode(cuda, b2q_mod, tmp_path):
    """The one-token expert-parallel layer with its reduction inside the kernel
    over peer memory (b2q_ep_peer_setup / _open) gives the same bits as the
    NCCL all-reduce path on every rank (all visible GPUs, at most 8), over nine
    calls of three layers (the exchange's epochs, both halves of its double
    buffer, and ranks holding none of a token's experts), and matches the
    single-GPU layer."""
    import torch

    world = min(torch.cuda.device_count(), 8)
    if world < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    path = str(tmp_path / "peer")
    env = dict(os.environ)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    try:
        mp.start_processes(_rank_peer, args=(world, _free_port(), path), nprocs=world, start_method="spawn",
                           join=True)
    finally:
        os.environ.clear()
        os.environ.update(env)
    outs = [np.load(path + f".{r}.npy") for r in range(world)]
    o0 = outs[0]
    for o in outs[1:]:
        assert np.array_equal(o0, o)
    if world <= 2:  # with more ranks NCCL may sum the partials in another order
        assert np.array_equal(o0[:9], o0[9:])  # peer path == NCCL path, bit for bit
    E, H, F, k = 16, 1024, 512, 4
    layers, wrs, xs = _peer_case(E, H, F, "cuda")
    for i in range(9):
        ref = b2q_mod.moe_decode(xs[i:i + 1], wrs[i % 3], layers[i % 3], k)
        assert rel_l2(_bf(o0[9 + i]), _bf(_np(ref))) < REL_L2
        assert rel_l2(_bf(o0[i]), _bf(_np(ref))) < REL_L2


# ---- all-to-all prefill ---------------------------------------------------------
def _emulate_a2a(x, wr, L, E, k, sizes):
    """Ranks emulated on one GPU through the three phase entry points: rank r owns
    the next sizes[r] tokens; blocks move between ranks by tensor copies in the
    order the NCCL exchange uses (senders in rank order)."""
    import torch

    from b2q.ep import a2a_combine, a2a_dispatch, a2a_experts, expert_range, shard_layer

    N = len(sizes)
    starts = np.cumsum([0] + list(sizes))
    disp = [a2a_dispatch(x[starts[r]:starts[r + 1]], wr, E, k, N) for r in range(N)]
    counts = [d[2].cpu().numpy() for d in disp]
    parts = []
    for d in range(N):
        rx = torch.cat([disp[s][0][d, :counts[s][d]] for s in range(N)])
        rm = torch.cat([disp[s][1][d, :counts[s][d]] for s in range(N)])
        lo, n = expert_range(E, N, d)
        parts.append(a2a_experts(rx, rm, shard_layer(L, lo, n), E, lo, k))
    outs = []
    for s in range(N):
        T_s = int(sizes[s])
        ret = torch.zeros((N, T_s, x.shape[1]), dtype=torch.float32, device=x.device)
        for d in range(N):
            off = int(sum(counts[q][d] for q in range(s)))
            ret[d, :counts[s][d]] = parts[d][off:off + counts[s][d]]
        outs.append(a2a_combine(ret, disp[s][3]))
    return torch.cat(outs), disp


def test_a2a_dispatch_plan_and_blocks(cuda, b2q_mod):
    import torch

    from b2q import synth
    from b2q.ep import a2a_dispatch
    from oracle.oracle import ep_a2a_plan

    E, H, k, N, T = 16, 1024, 4, 3, 70
    wr = synth.router_weight(E, H, seed=91)
    x = synth.activations((T, H), seed=93)
    send_x, send_meta, counts, pos, idx, w = a2a_dispatch(x, wr, E, k, N)
    torch.cuda.synchronize()
    _, ref_idx = b2q_mod.moe_prefill(x, wr, synth.moe_layer(E, H, 512, 64, seed=90), k, return_routing=True)[:2]
    assert np.array_equal(_np(idx).astype(np.uint32), _np(ref_idx).astype(np.uint32))
    rpos, rcounts = ep_a2a_plan(_np(idx).astype(np.uint32), E, N)
    assert np.array_equal(_np(pos), rpos) and np.array_equal(_np(counts), rcounts)
    xs, sx, sm = _np(x), _np(send_x), _np(send_meta).view(np.uint32)
    for d in range(N):
        rows = [t for t in range(T) if rpos[t, d] >= 0]
        assert np.array_equal(sx[d, :len(rows)], xs[rows])
        assert np.array_equal(sm[d, :len(rows), :k], _np(idx).view(np.uint32)[rows])
        assert np.array_equal(sm[d, :len(rows), k:], _np(w).view(np.uint32)[rows])


@pytest.mark.parametrize("sizes", [(48, 48), (40, 0, 56), (10, 30, 1, 55), (12, 12, 0, 12, 12, 24, 12, 12)])
def test_a2a_emulated_ranks_match_the_layer(cuda, b2q_mod, oracle, sizes):
    E, H, F, k = 16, 1024, 512, 4
    L, wr = _layer(E, H, F, 90)
    from b2q import synth

    x = synth.activations((sum(sizes), H), seed=94)
    out, _ = _emulate_a2a(x, wr, L, E, k, sizes)
    ref = b2q_mod.moe_prefill(x, wr, L, k)
    assert rel_l2(_bf(_np(out)), _bf(_np(ref))) < 5e-3
    lg = b2q_mod.router_logits(x, wr)
    ridx, rw = oracle.route(_np(lg), k)
    rows = list(range(0, sum(sizes), 11))
    ro = _bf(oracle.moe_experts_prefill(_np(x), ridx, rw, {kk: _np(v) for kk, v in L.items()}, k, rows=rows))
    assert rel_l2(_bf(_np(out))[rows], ro) < REL_L2


def test_a2a_single_rank_call(cuda, b2q_mod):
    """One rank (no communicator): the chained call equals the phases bit for bit,
    and a second call with the workspace reused gives the same output."""
    from b2q import synth
    from b2q.ep import EPMoE

    E, H, F, k, T = 16, 1024, 512, 4, 80
    L, wr = _layer(E, H, F, 90)
    x = synth.activations((T, H), seed=95)
    moe = EPMoE(wr, L, E, 0, k)
    a = moe.prefill_a2a(x, T_max=96)
    b = moe.prefill_a2a(x, T_max=96)
    ref, _ = _emulate_a2a(x, wr, L, E, k, [T])
    assert np.array_equal(_np(a), _np(ref)) and np.array_equal(_np(a), _np(b))


def _rank_a2a(rank, world, port, T, path):
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import sys

        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        sys.path[:0] = [root, os.path.join(root, "mlxfast-qwen38-125b-a6b-engine_b200")]
        from b2q import synth
        from b2q.ep import EPComm, EPMoE, expert_range, shard_layer, token_range

        E, H, F, k = 16, 1024, 512, 4
        L = synth.moe_layer(E, H, F, 64, device="cuda", seed=90)
        wr = synth.router_weight(E, H, device="cuda", seed=91)
        x = synth.activations((T, H), device="cuda", seed=96)
        comm = EPComm(world, rank)
        lo, n = expert_range(E, world, rank)
        t_lo, t_n = token_range(T, world, rank)
        moe = EPMoE(wr, shard_layer(L, lo, n), E, lo, k, comm)
        T_max = max(token_range(T, world, r)[1] for r in range(world))
        out = moe.prefill_a2a(x[t_lo:t_lo + t_n], T_max=T_max)
        torch.cuda.synchronize()
        np.save(path + f".{rank}.npy", _np(out))
        comm.close()
    finally:
        dist.destroy_process_group()


def test_two_ranks_nccl_a2a(cuda, b2q_mod, tmp_path):
    """Two GPUs over NCCL: the same bits as the one-GPU emulation of the two ranks."""
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    from b2q import synth
    from b2q.ep import token_range

    T = 97
    path = str(tmp_path / "a2a")
    env = dict(os.environ)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    try:
        mp.start_processes(_rank_a2a, args=(2, _free_port(), T, path), nprocs=2, start_method="spawn", join=True)
    finally:
        os.environ.clear()
        os.environ.update(env)
    got = np.concatenate([np.load(path + f".{r}.npy") for r in range(2)])
    E, H, F, k = 16, 1024, 512, 4
    L, wr = synth.moe_layer(E, H, F, 64, seed=90), synth.router_weight(E, H, seed=91)
    x = synth.activations((T, H), seed=96)
    ref, _ = _emulate_a2a(x, wr, L, E, k, [token_range(T, 2, r)[1] for r in range(2)])
    assert np.array_equal(got, _np(ref))
