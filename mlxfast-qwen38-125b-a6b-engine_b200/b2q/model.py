"""A generic 4-bit MoE decoder built around the path (the full-model configs).

The reference's model (Qwen3.8-class, mlx-swift-lm's Qwen4ExpModel) has
attention variants, hyper-connections and other blocks that are outside the
path; this decoder is the generic shape the benchmark configuration names:

    h = embed(tokens)                                  4-bit tied table
    per layer:
        a   = rms_norm(h) ; q|k|v = QuantizedLinear(a)  one fused 4-bit product
        q,k = rope(q, k)   (non-interleaved, theta)     ; k, v -> bf16 KV cache
        h  += QuantizedLinear_o(attention(q, K, V))     GQA, causal
        h  += MoE(rms_norm(h))                          router top-k, SwiGLU experts
    logits = lm_head(rms_norm(h))                       the tied table as a 4-bit product
    MTP draft (one extra block, DeepSeek-style): x = eh_proj([norm(embed(t+1)) ; norm(h_t)]),
        one block, the shared final norm and lm_head -> the token after next

Every weight product and the MoE layers run through the library (qmv / qmm,
the fused decode MoE, the sorted prefill MoE); RMSNorm, RoPE and the token
embedding are library kernels too. Attention itself is PyTorch's SDPA on the
GPU for prefill (outside the path); windows of up to 8 rows (decode, MTP
verify) use the library's GQA decode attention, which reads the rows'
positions on the device. The residual add is fused into the following norm.
A greedy decode step can be captured in a CUDA graph (`Decoder.decode_graph`):
token id and position live in device buffers that the graph updates itself,
so one replay is one token.

Random-init weights follow the synthetic distributions of the benchmark
(packed nibbles uniform, scales U(0.002, 0.02), biases -8*scale + N(0, 1e-3)).
"""
from __future__ import annotations

import dataclasses

import torch
import torch.nn.functional as Fnn

from . import ops, synth
from ._lib import check, lib
from .ep import EPMoE, expert_range, shard_layer
from .nn import MoE, QuantizedLinear


@dataclasses.dataclass
class DecoderConfig:
    n_layers: int = 48
    hidden: int = 4096
    n_heads: int = 32
    n_kv_heads: int = 4
    head_dim: int = 128
    n_experts: int = 128
    top_k: int = 8
    expert_ffn: int = 1536
    vocab: int = 151936
    rope_theta: float = 1e6
    rms_eps: float = 1e-6
    group_size: int = 64
    mtp: bool = True
    max_seq: int = 2048

    def validate(self):
        if self.n_heads % self.n_kv_heads:
            raise ValueError("n_heads must be a multiple of n_kv_heads")
        if self.head_dim % 2 or self.hidden % 8:
            raise ValueError("head_dim must be even and hidden a multiple of 8")
        if self.top_k > self.n_experts:
            raise ValueError("top_k > n_experts")
        return self

    @property
    def qkv_rows(self) -> int:
        return (self.n_heads + 2 * self.n_kv_heads) * self.head_dim

    def packed_bytes(self, rows: int, K: int) -> int:
        """Bytes of a 4-bit matrix: packed nibbles + bf16 scale and bias per group."""
        return rows * (K // 2 + 2 * 2 * (K // self.group_size))

    def decode_bytes_per_token(self, position: int) -> int:
        """Weight + KV bytes one greedy decode step reads (no MTP): per layer the
        attention projections, the router, k experts, the KV cache up to `position`;
        then the lm_head."""
        H, hd = self.hidden, self.head_dim
        attn = self.packed_bytes(self.qkv_rows, H) + self.packed_bytes(H, self.n_heads * hd)
        expert = 2 * self.packed_bytes(self.expert_ffn, H) + self.packed_bytes(H, self.expert_ffn)
        router = self.n_experts * H * 2
        kv = 2 * self.n_kv_heads * hd * 2 * (position + 1)
        return self.n_layers * (attn + router + self.top_k * expert + kv) + self.packed_bytes(self.vocab, H)


def _ql(rows, K, gs, dev, seed):
    w, s, b = synth.packed_weights((rows,), K, gs, dev, seed)
    return QuantizedLinear(w, s, b, gs, 4)


def _norm_weight(H, dev, seed):
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    return (1.0 + 0.05 * torch.randn(H, generator=g, device=dev)).to(torch.bfloat16)


class Block:
    """One decoder block: attention (fused q|k|v product, RoPE, GQA) then the MoE.

    The residual stream is carried as (h, delta): a block adds the previous
    block's MoE output into h inside its first norm (b2q_add_rms_norm) and
    returns its own MoE output as the next delta."""

    def __init__(self, cfg: DecoderConfig, dev, seed: int, status: torch.Tensor, attn_ws: torch.Tensor,
                 ep: tuple | None = None):
        H, hd = cfg.hidden, cfg.head_dim
        self.cfg = cfg
        self.attn_norm = _norm_weight(H, dev, seed)
        self.qkv = _ql(cfg.qkv_rows, H, cfg.group_size, dev, seed + 1)
        self.o = _ql(H, cfg.n_heads * hd, cfg.group_size, dev, seed + 2)
        self.mlp_norm = _norm_weight(H, dev, seed + 3)
        router = synth.router_weight(cfg.n_experts, H, dev, seed + 4)
        experts = synth.moe_layer(cfg.n_experts, H, cfg.expert_ffn, cfg.group_size, dev, seed + 5)
        if ep is None:
            self.moe = MoE(router, experts, cfg.top_k, cfg.group_size)
        else:
            # expert parallel: this rank keeps its contiguous block of experts; the
            # layer output is the NCCL all-reduce of the ranks' fp32 partials
            comm, world, rank = ep
            lo, n = expert_range(cfg.n_experts, world, rank)
            local = shard_layer(experts, lo, n)
            del experts
            self.moe = EPMoE(router, local, cfg.n_experts, lo, cfg.top_k, comm, cfg.group_size)
        self.k_cache = torch.zeros((cfg.max_seq, cfg.n_kv_heads, hd), dtype=torch.bfloat16, device=dev)
        self.v_cache = torch.zeros_like(self.k_cache)
        self.status, self.attn_ws = status, attn_ws
        # one-token steps with the norms fused into the products (the plain MoE;
        # the expert-parallel layer keeps the separate norm)
        self._fused_norm = ep is None

    def _decode_one(self, h: torch.Tensor, delta, positions):
        """One token: norm + q|k|v in one launch, attention, o, norm + MoE in one
        launch. None when a fused call is outside its kernel (the separate path
        is taken and this block stops trying)."""
        cfg = self.cfg
        st = ops._stream(h.device)
        q = self.qkv
        h2 = torch.empty_like(h) if delta is not None else h
        qkv = torch.empty((1, cfg.qkv_rows), dtype=torch.bfloat16, device=h.device)
        rc = lib().b2q_qmv_norm(h.data_ptr(), None if delta is None else delta.data_ptr(), self.attn_norm.data_ptr(),
                                cfg.rms_eps, None if delta is None else h2.data_ptr(), q.weight.data_ptr(),
                                q.scales.data_ptr(), q.biases.data_ptr(), qkv.data_ptr(), cfg.qkv_rows, cfg.hidden,
                                q.group_size, q.bits, st)
        if rc == -2:  # B2Q_EUNSUPPORTED
            self._fused_norm = False
            return None
        check(rc)
        o = self.o(self._attend(qkv, positions))
        h3 = torch.empty_like(h)
        out = self.moe.decode_norm(h2, o, self.mlp_norm, cfg.rms_eps, h3)
        if out is None:
            self._fused_norm = False
            m = add_rms_norm(h2, o, self.mlp_norm, cfg.rms_eps)
            return h2, self.moe(m)
        return h3, out

    def attention(self, a: torch.Tensor, positions: torch.Tensor, pos0: int | None = None) -> torch.Tensor:
        """a [T, H] normed -> attention output [T, n_heads * hd] (bf16).

        positions: int32 [T] device tensor of the rows' positions (consecutive).
        Windows of up to 8 rows (decode, verify) attend through b2q_attn_decode
        (rope, KV append and attention in one launch), which reads the positions
        on the device (graph-safe); longer windows
        (prefill) use the framework's causal attention from row pos0 on."""
        return self._attend(self.qkv(a), positions, pos0)

    def _attend(self, qkv: torch.Tensor, positions: torch.Tensor, pos0: int | None = None) -> torch.Tensor:
        """The attention of `attention` from the fused q|k|v rows [T, (nq + 2 nk) hd]."""
        cfg = self.cfg
        T = qkv.shape[0]
        nq, nk, hd = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
        a = qkv
        st = ops._stream(a.device)
        if T <= 8:
            # rope, KV append, attention and the chunk merge in one launch
            out = torch.empty((T, nq * hd), dtype=torch.bfloat16, device=a.device)
            check(lib().b2q_attn_decode(qkv.data_ptr(), cfg.qkv_rows, positions.data_ptr(), self.k_cache.data_ptr(),
                                        self.v_cache.data_ptr(), out.data_ptr(), T, nq, nk, hd, cfg.rope_theta,
                                        cfg.max_seq, self.status.data_ptr(), self.attn_ws.data_ptr(),
                                        self.attn_ws.numel(), st))
            return out
        check(lib().b2q_rope_kv(qkv.data_ptr(), T, nq, nk, hd, positions.data_ptr(), cfg.rope_theta,
                                self.k_cache.data_ptr(), self.v_cache.data_ptr(), cfg.max_seq,
                                self.status.data_ptr(), st))
        if pos0 is None:
            raise ValueError("a window of more than 8 rows needs its first position on the host")
        L = pos0 + T
        qh = qkv[:, :nq * hd].view(T, nq, hd).permute(1, 0, 2).unsqueeze(0)
        kh = self.k_cache[:L].permute(1, 0, 2).unsqueeze(0)
        vh = self.v_cache[:L].permute(1, 0, 2).unsqueeze(0)
        if pos0 == 0:
            o = Fnn.scaled_dot_product_attention(qh, kh, vh, is_causal=True, enable_gqa=True)
        else:
            qi = torch.arange(pos0, pos0 + T, device=a.device).view(T, 1)
            ki = torch.arange(L, device=a.device).view(1, L)
            m = torch.zeros((T, L), dtype=torch.bfloat16, device=a.device).masked_fill(ki > qi, float("-inf"))
            o = Fnn.scaled_dot_product_attention(qh, kh, vh, attn_mask=m, enable_gqa=True)
        return o.squeeze(0).permute(1, 0, 2).reshape(T, nq * hd).contiguous()

    def __call__(self, h: torch.Tensor, delta, positions, pos0=None):
        """(h, delta) -> (h + delta + attention, MoE output). Windows of several
        rows update h in place; one-token steps return a new residual tensor
        (the norms are fused into the q|k|v product and the MoE kernel, whose
        CTAs all read h while one of them writes the sum)."""
        cfg = self.cfg
        if h.shape[0] == 1 and self._fused_norm:
            r = self._decode_one(h, delta, positions)
            if r is not None:
                return r
        a = add_rms_norm(h, delta, self.attn_norm, cfg.rms_eps)
        o = self.o(self.attention(a, positions, pos0))
        m = add_rms_norm(h, o, self.mlp_norm, cfg.rms_eps)
        return h, self.moe(m)


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    x = x.contiguous()
    T, H = x.shape
    out = torch.empty_like(x)
    check(lib().b2q_rms_norm(x.data_ptr(), w.data_ptr(), out.data_ptr(), T, H, eps, ops._stream(x.device)))
    return out


def add_rms_norm(h: torch.Tensor, delta, w: torch.Tensor, eps: float) -> torch.Tensor:
    """h += delta (bf16, in place; skipped when delta is None), then rms_norm(h)."""
    T, H = h.shape
    out = torch.empty_like(h)
    check(lib().b2q_add_rms_norm(h.data_ptr(), None if delta is None else delta.data_ptr(), w.data_ptr(),
                                 h.data_ptr(), out.data_ptr(), T, H, eps, ops._stream(h.device)))
    return out


class Decoder:
    """Random-init decoder of `cfg` on `device` (seeded), with a bf16 KV cache of cfg.max_seq rows per layer.

    expert_parallel=(comm, world, rank) shards every MoE layer's experts over the
    ranks of `comm` (an EPComm, or None for one rank): attention, norms, router
    and embeddings stay replicated, every rank runs the same token stream, and
    each MoE layer ends in one NCCL all-reduce of the fp32 layer partial (the
    expert-parallel full-model configuration). All ranks must call the same
    methods in the same order."""

    def __init__(self, cfg: DecoderConfig, device="cuda", seed: int = 0, expert_parallel: tuple | None = None):
        self.cfg = cfg.validate()
        dev = torch.device(device)
        self.device = dev
        H = cfg.hidden
        ew, es, eb = synth.packed_weights((cfg.vocab,), H, cfg.group_size, dev, seed)
        self.embed_w, self.embed_s, self.embed_b = ew, es, eb
        self.lm_head = QuantizedLinear(ew, es, eb, cfg.group_size, 4)  # tied
        self._status = torch.zeros(1, dtype=torch.int32, device=dev)
        ws = lib().b2q_attn_decode_workspace_size(8, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.max_seq)
        self._attn_ws = torch.zeros(ws, dtype=torch.uint8, device=dev)  # chunk counters start at zero
        self.blocks = [Block(cfg, dev, seed + 100 * (i + 1), self._status, self._attn_ws, expert_parallel)
                       for i in range(cfg.n_layers)]
        self.final_norm = _norm_weight(H, dev, seed + 7)
        self.mtp = None
        if cfg.mtp:
            base = seed + 100 * (cfg.n_layers + 1)
            self.mtp = {"enorm": _norm_weight(H, dev, base), "hnorm": _norm_weight(H, dev, base + 1),
                        "eh_proj": _ql(H, 2 * H, cfg.group_size, dev, base + 2),
                        "block": Block(cfg, dev, base + 10, self._status, self._attn_ws, expert_parallel)}
        self._graph = None

    # ---- pieces --------------------------------------------------------------
    def embed(self, ids: torch.Tensor) -> torch.Tensor:
        ids = ids.to(torch.int32).contiguous().view(-1)
        T = ids.numel()
        out = torch.empty((T, self.cfg.hidden), dtype=torch.bfloat16, device=self.device)
        check(lib().b2q_embed_gather(self.embed_w.data_ptr(), self.embed_s.data_ptr(), self.embed_b.data_ptr(),
                                     ids.data_ptr(), out.data_ptr(), T, self.cfg.vocab, self.cfg.hidden,
                                     self.cfg.group_size, 4, self._status.data_ptr(), ops._stream(self.device)))
        return out

    def logits(self, h: torch.Tensor) -> torch.Tensor:
        return self.lm_head(rms_norm(h, self.final_norm, self.cfg.rms_eps))

    def status(self) -> int:
        """Device-side error recorded by the embedding lookup (B2Q_EINVAL for a bad token id), then cleared."""
        v = int(self._status.item())
        self._status.zero_()
        return v

    # ---- eager forward ---------------------------------------------------------
    def forward(self, ids: torch.Tensor, pos0: int = 0):
        """Tokens ids [T] at positions pos0.. -> (hidden [T, H] after the last block, logits of the last row)."""
        T = ids.numel()
        if pos0 + T > self.cfg.max_seq:
            raise ValueError("sequence longer than max_seq")
        positions = torch.arange(pos0, pos0 + T, dtype=torch.int32, device=self.device)
        h, normed = self._blocks(self.embed(ids), positions, pos0)
        return h, self.lm_head(normed[-1:])

    def _blocks(self, h, positions, pos0=None, blocks=None):
        """Rows through the blocks; returns (final residual h, final-normed h)."""
        delta = None
        for blk in (self.blocks if blocks is None else blocks):
            h, delta = blk(h, delta, positions, pos0)
        normed = add_rms_norm(h, delta, self.final_norm, self.cfg.rms_eps)
        return h, normed

    def mtp_draft(self, h_prev: torch.Tensor, ids: torch.Tensor, pos0: int) -> torch.Tensor:
        """The draft head over rows pos0..: row p takes the main model's hidden of
        position p - 1 (h_prev[i]) and the token at p (ids[i]); it appends row p to
        the head's own KV cache and returns the logits of the last row, a guess of
        the token at p + 1."""
        m = self.mtp
        e = rms_norm(self.embed(ids), m["enorm"], self.cfg.rms_eps)
        hh = rms_norm(h_prev.contiguous(), m["hnorm"], self.cfg.rms_eps)
        x = m["eh_proj"](torch.cat([e, hh], dim=-1))
        positions = torch.arange(pos0, pos0 + x.shape[0], dtype=torch.int32, device=self.device)
        _, normed = self._blocks(x, positions, pos0, blocks=[m["block"]])
        return self.lm_head(normed[-1:])

    def generate(self, prompt: torch.Tensor, n_new: int, use_mtp: bool = False):
        """Greedy decode (eager). With use_mtp the draft head proposes the token after
        next and a two-row window verifies it (accepted when the main model agrees).
        Returns (tokens [n_new] on the host, accepted draft count)."""
        prompt = prompt.to(self.device).view(-1)
        T = prompt.numel()
        h, lg = self.forward(prompt, 0)
        out = [int(lg.argmax(-1).item())]
        pos = T  # position of out[-1]
        h_last = h[-1:]
        accepted = 0
        use_mtp = use_mtp and self.mtp is not None
        if use_mtp:
            # the head's cache over the prompt: row p from (h_{p-1}, token p), h_{-1} = 0
            hp = torch.cat([torch.zeros_like(h[:1]), h[:-1]])
            self.mtp_draft(hp, prompt, 0)
        while len(out) < n_new:
            tok = torch.tensor([out[-1]], dtype=torch.int32, device=self.device)
            if use_mtp and pos + 2 <= self.cfg.max_seq:
                draft = int(self.mtp_draft(h_last, tok, pos).argmax(-1).item())
                ids = torch.tensor([out[-1], draft], dtype=torch.int32, device=self.device)
                hw = self._window(ids, pos)
                lw = self.logits(hw)
                a0 = int(lw[0].argmax(-1).item())
                if a0 == draft:
                    accepted += 1
                    out += [draft, int(lw[1].argmax(-1).item())]
                    # the head's row pos + 1 (the accepted draft) before it drafts from pos + 2
                    self.mtp_draft(hw[0:1], ids[1:2], pos + 1)
                    h_last = hw[1:2]
                    pos += 2
                else:
                    out.append(a0)
                    h_last = hw[0:1]
                    pos += 1
            else:
                hw = self._window(tok, pos)
                out.append(int(self.logits(hw).argmax(-1).item()))
                h_last = hw
                pos += 1
        return out[:n_new], accepted

    def _window(self, ids: torch.Tensor, pos0: int) -> torch.Tensor:
        positions = torch.arange(pos0, pos0 + ids.numel(), dtype=torch.int32, device=self.device)
        h, _ = self._blocks(self.embed(ids), positions, pos0)
        return h

    # ---- CUDA-graph decode ----------------------------------------------------------
    def decode_graph(self):
        """Capture one greedy decode step: the graph reads the token and position
        from device buffers, appends to the KV cache, writes the argmax back as the
        next token and advances the position (positions up to max_seq - 1).
        Returns (replay_fn, token_buf, pos_buf, logits_buf); logits_buf holds the
        last replayed step's logits [1, vocab]."""
        cfg = self.cfg
        dev = self.device
        tok = torch.zeros(1, dtype=torch.int32, device=dev)
        pos = torch.zeros(1, dtype=torch.int32, device=dev)
        lg_buf = torch.zeros((1, cfg.vocab), dtype=torch.bfloat16, device=dev)
        stream = torch.cuda.Stream(device=dev)

        def step():
            _, normed = self._blocks(self.embed(tok), pos)
            lg = self.lm_head(normed)
            lg_buf.copy_(lg)
            tok.copy_(lg.argmax(-1).to(torch.int32).view(1))
            pos.add_(1)

        # warm the library's per-shape state (tensor maps, attributes) outside the
        # capture; the warm-up writes KV row max_seq - 1, which no caller has yet
        tok.zero_()
        pos.fill_(cfg.max_seq - 1)
        stream.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(stream):
            step()
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            step()
        torch.cuda.synchronize(dev)
        self._graph = graph

        def replay():
            graph.replay()

        return replay, tok, pos, lg_buf
