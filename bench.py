"""Benchmark of the affine 4-bit MoE hot path on B200.

Workload (N = 1): config 1 of the spec -- one MoE layer decoding one token
(H 4096, 128 experts, top-8, expert F 1536, 4-bit g64), synthetic seeded
inputs. A step is one full layer for one token (router, routing, gate|up +
SwiGLU, down + weighted combine). To keep the selected experts cold in L2,
steps rotate over 8 independent layers (10.9 GB of expert weights) and a fresh
token per step. Config 2 (prefill, 2048 tokens) is reported under "prefill".

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b2q|reference]

Prints ONE JSON line on rank 0.
"""
from __future__ import annotations

import argparse
import json
import multiprocessing as mp
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "mlxfast-qwen38-125b-a6b-engine_b200")
for _p in (ROOT, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

H, E, F, TOPK, GS = 4096, 128, 1536, 8, 64
PREFILL_T = 2048
N_LAYERS = 8
N_TOKENS = 4096
# Algorithmic bytes of one decode step (8 experts x (gate + up + down) packed
# weights with scales/biases, the bf16 router, activations): 86,049,344 B.
# Activations: x and the output row (2 x 8,192), the SwiGLU rows written and
# read back (2 x 8 x 1536 x 2), the router logits (512) and the selected
# experts with their weights (64): 66,112 B.
EXPERT_BYTES = 3 * (F * (H // 2 + 2 * 2 * H // GS))  # gate/up/down are the same size here
ACT_BYTES = 2 * H * 2 + 2 * TOPK * F * 2 + E * 4 + TOPK * 4 * 2
DECODE_BYTES = TOPK * EXPERT_BYTES + E * H * 2 + ACT_BYTES
PREFILL_FLOP = PREFILL_T * TOPK * (2 * 2 * F * H + 2 * H * F) + 2 * PREFILL_T * E * H
METRIC = "decode tok/s (bs=1) + gather_qmv HBM GB/s and % of 8 TB/s; prefill tok/s"
WORKLOAD = "config 1: one MoE layer decode, bs=1, H4096 E128 top8 F1536 4-bit g64"


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d.get("hbm_gbs", 6650.0), d.get("bf16_tflops", 1590.0), "measured"
    return 6650.0, 1590.0, "fallback"


def load_traffic(name):
    """ncu DRAM bytes per launch recorded in profiles/<name>.json (or None)."""
    p = os.path.join(ROOT, "profiles", name)
    if os.path.exists(p):
        try:
            return json.load(open(p)).get("dram_bytes_per_launch")
        except Exception:
            return None
    return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.proc = None
        self.path = os.path.join("/tmp", f"b2q_clocks_{os.getpid()}.csv")

    def __enter__(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=self.f, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.f.close()

    def summary(self):
        if self.proc is None or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        for line in open(self.path):
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), float(parts[3]), parts[5:9]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i, v in enumerate(r[3]) if v.lower() == "active"})
        loaded = [r[0] for r in rows if r[2] > 200.0] or [r[0] for r in rows]
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": max(r[1] for r in rows), "reasons": reasons,
                "samples": len(rows), "power_w_max": max(r[2] for r in rows)}


# --------------------------------------------------------------------------
# CPU baselines (the reference's own MLX CPU quantized kernels)
# --------------------------------------------------------------------------
_REF_STATE = {}


def _ref_init(seed, rows):
    """Pool initializer: build one process's weight rows once (outside any timing)."""
    import numpy as np

    from oracle.oracle import MlxRef, Oracle, bf16_to_f32, f32_to_bf16

    rng = np.random.default_rng(seed)
    K = H
    wq = rng.integers(0, 2**32, size=(rows, K // 8), dtype=np.uint64).astype(np.uint32)
    s = f32_to_bf16(rng.uniform(0.002, 0.02, (rows, K // GS)).astype(np.float32))
    b = f32_to_bf16(-8.0 * bf16_to_f32(s) + rng.normal(0, 1e-3, s.shape).astype(np.float32))
    x = f32_to_bf16(rng.standard_normal((1, K)).astype(np.float32))
    _REF_STATE.update(ref=MlxRef() if MlxRef.available() else None, orc=Oracle(), wq=wq, s=s, b=b, x=x,
                      out=np.zeros((1, rows), np.uint16))


def _ref_run(reps):
    """Time `reps` passes of this process's rows through the MLX CPU kernel (seconds)."""
    st = _REF_STATE
    t0 = time.perf_counter()
    for _ in range(reps):
        if st["ref"] is not None:
            st["ref"].qmm(st["x"], st["wq"], st["s"], st["b"], GS, 4, out=st["out"])
        else:
            st["orc"].qmm_mlx_cpu(st["x"], st["wq"], st["s"], st["b"], GS, 4)
    return time.perf_counter() - t0


def _ref_worker(args):
    seed, rows, reps = args
    _ref_init(seed, rows)
    return _ref_run(reps)


def cpu_row_cost():
    """Seconds per 4096-element qmm row on one core (reference kernel)."""
    rows = 256
    t = _ref_worker((0, rows, 3))
    return t / (3 * rows)


def decode_rows_per_token():
    # gate/up: 2 x 1536 rows of K = 4096; down: 4096 rows of K = 1536 = 1536 rows of K = 4096 equivalent
    return TOPK * (2 * F + H * F // H)


def prefill_rows_per_assignment():
    # gate + up: 2 x 1536 rows of K = 4096; down: 4096 rows of K = 1536 = 1536 rows of K = 4096 equivalent
    return 2 * F + H * F // H


def prefill_cpu_baseline(t_row, kind):
    """Config 2 on one core, extrapolated from the measured row cost of the reference
    kernel: the reference's CPU gather runs one qmm call per (token, expert) pair
    (backend/cpu/quantized.cpp:701-747), so a prefill layer is 2048 x 8 assignments
    of 4608 K=4096 row-equivalents plus the router (128 rows per token)."""
    rows = PREFILL_T * TOPK * prefill_rows_per_assignment() + PREFILL_T * E
    sec = rows * t_row
    return {"value": PREFILL_T / sec, "unit": "tok/s", "cores": 1, "kind": kind,
            "sample": (f"extrapolated: measured per-row time of the reference's MLX CPU kernel (K=4096 4-bit g64, "
                       f"bf16 sum) x {rows} row-equivalents per 2048-token layer (16384 assignments x "
                       f"{prefill_rows_per_assignment()} + router); SwiGLU, sort and combine omitted")}


# config 3 shape (the defaults of b2q.model.DecoderConfig)
DEC_LAYERS, DEC_QKV_ROWS, DEC_ATTN_DIM, DEC_VOCAB = 48, (32 + 2 * 4) * 128, 32 * 128, 151936


def decoder_rows_per_token(n_layers=DEC_LAYERS):
    """K=4096 row-equivalents of the 4-bit products one decode token runs: per
    layer q|k|v (5120 rows), o (4096 rows of K = 4096) and the k experts; then
    the tied lm_head (151,936 rows)."""
    return n_layers * (DEC_QKV_ROWS + H * DEC_ATTN_DIM // 4096 + decode_rows_per_token()) + DEC_VOCAB


def decoder_cpu_baseline(t_row, kind, n_layers=DEC_LAYERS):
    """Config 3 on one core, lower bound (quantized share only): the measured row
    cost of the reference kernel times the 4-bit rows of one token; attention,
    norms, the bf16 router and sampling are left out."""
    rows = decoder_rows_per_token(n_layers)
    return {"value": 1.0 / (rows * t_row), "unit": "tok/s", "cores": 1, "kind": kind,
            "sample": (f"lower bound, quantized share only, extrapolated: measured per-row time of the reference's "
                       f"MLX CPU kernel (K=4096 4-bit g64, bf16 sum) x {rows} row-equivalents per token "
                       f"({n_layers} layers x (q|k|v {DEC_QKV_ROWS} + o {DEC_ATTN_DIM} + {TOPK} experts "
                       f"{decode_rows_per_token()}) + lm_head {DEC_VOCAB}); attention, norms, router and "
                       f"sampling omitted")}


def cpu_baseline_sample(budget_s=12.0):
    """Single core, the reference CPU kernel, bounded sample of config 1."""
    from oracle.oracle import MlxRef

    kind = "reference" if MlxRef.available() else "port"
    t_row = cpu_row_cost()
    rows = max(64, min(4096, int(budget_s / 3 / t_row)))
    t = _ref_worker((1, rows, 3))
    per_row = t / (3 * rows)
    tok_s = 1.0 / (per_row * decode_rows_per_token())
    sample = (f"{3 * rows} rows of K=4096 4-bit g64 qmv through the reference's MLX CPU kernel "
              f"(backend/cpu/quantized.cpp _qmm_t, bf16 sum) on 1 core; tok/s = 1/(row time x "
              f"{decode_rows_per_token()} row-equivalents per token); router/SwiGLU/combine (<2% of work) omitted")
    return {"value": tok_s, "unit": "tok/s", "cores": 1, "kind": kind, "sample": sample, "row_s": per_row}


def run_reference(args, rank, world):
    if rank != 0:
        return
    from oracle.oracle import MlxRef

    kind = "reference" if MlxRef.available() else "port"
    cores = os.cpu_count() or 1
    t_row = cpu_row_cost()
    total_steps = args.steps + args.warmup
    budget = 60.0  # seconds of kernel time over the whole run
    rows = max(1, int(budget / max(1, total_steps) / t_row))
    ctx = mp.get_context("spawn")
    pools = [ctx.Pool(1, initializer=_ref_init, initargs=(i, rows)) for i in range(cores)]
    try:
        for _ in range(args.warmup):
            [r.get() for r in [p.apply_async(_ref_run, (1,)) for p in pools]]
        dt = 0.0
        for _ in range(args.steps):
            # a step ends when the slowest process has done its rows
            dt += max(r.get() for r in [p.apply_async(_ref_run, (1,)) for p in pools])
    finally:
        for p in pools:
            p.terminate()
    tok = args.steps * cores * rows / decode_rows_per_token()
    value = tok / dt
    sample = (f"each step: {cores} processes x {rows} K=4096 rows of the reference MLX CPU 4-bit kernel "
              f"(backend/cpu/quantized.cpp), throughput converted at {decode_rows_per_token()} row-equivalents "
              "per decode token")
    line = {"metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1000.0 * dt / max(1, args.steps), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded)",
            "config": {"workload": WORKLOAD, "parallelism": f"host CPU, {cores} processes of the reference kernel"},
            "impl": "reference",
            "cpu_baseline": {"value": value, "unit": "tok/s", "cores": cores, "kind": kind, "sample": sample},
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------
# GPU arm
# --------------------------------------------------------------------------
DEC_PROMPT, DEC_NEW = 1024, 256


def run_decoder(dev, hbm_peak, peak_kind, n_new=DEC_NEW, prefill_warmup=2, n_layers=48):
    """Config 3: random-init 48-layer decoder; prefill 1024 random ids, then 256 greedy
    tokens, each one replay of the captured decode step."""
    import torch

    from b2q.model import Decoder, DecoderConfig

    cfg = DecoderConfig(max_seq=DEC_PROMPT + DEC_NEW, n_layers=n_layers)
    dec = Decoder(cfg, device=dev, seed=11)
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    prompt = torch.randint(0, cfg.vocab, (DEC_PROMPT,), generator=g, device=dev, dtype=torch.int32)
    try:
        replay, tok, pos, lg = dec.decode_graph()
    except Exception as ex:  # reported, not hidden: the leg then has no decode number
        return {"workload": "config 3", "error": f"decode step capture failed: {ex!r}"[:300]}
    for _ in range(prefill_warmup):
        dec.forward(prompt, 0)
    torch.cuda.synchronize(dev)
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p0.record()
    _, logits = dec.forward(prompt, 0)
    p1.record()
    torch.cuda.synchronize(dev)
    prefill_ms = p0.elapsed_time(p1)
    tok.copy_(logits.argmax(-1).to(torch.int32).view(1))
    pos.fill_(DEC_PROMPT)
    tokens = torch.empty(n_new, dtype=torch.int32, device=dev)
    tokens[0].copy_(tok[0])
    torch.cuda.synchronize(dev)
    d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    d0.record()
    for i in range(1, n_new):
        replay()
        tokens[i].copy_(tok[0])
    d1.record()
    torch.cuda.synchronize(dev)
    steps = n_new - 1
    ms_tok = d0.elapsed_time(d1) / steps
    status = dec.status()
    bytes_tok = cfg.decode_bytes_per_token(DEC_PROMPT + n_new // 2)
    gbs = bytes_tok / (ms_tok * 1e-3) / 1e9
    out = {"workload": f"config 3: {n_layers}-layer 4-bit MoE decoder (H4096, GQA 32/4 x 128, E128 top8 F1536, vocab 151936 "
                       f"tied 4-bit), random init, prompt {DEC_PROMPT} random ids then {n_new} greedy tokens",
           "decode_tok_s": 1000.0 / ms_tok, "ms_per_token": ms_tok, "prefill_tok_s": DEC_PROMPT * 1000.0 / prefill_ms,
           "prefill_ms": prefill_ms, "bytes_per_token": bytes_tok,
           "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm_peak, "unit": "GB/s", "frac": gbs / hbm_peak,
                        "peak_kind": peak_kind},
           "decode_form": "one CUDA-graph replay per token (graph updates token and position on the device)",
           "mtp": "draft head built; greedy timing without speculation (random weights never agree)",
           "device_status": status, "distinct_tokens": int(torch.unique(tokens).numel())}
    del dec, replay
    torch.cuda.empty_cache()
    return out


C0_COPIES, C0_CALLS = 32, 256
C0_BYTES = 4096 * (4096 // 2 + 2 * 2 * 4096 // GS) + 2 * 4096 + 2 * 4096  # 9,453,568 B per call


def run_c0(dev, stream, hbm_peak, peak_kind):
    """Config 0: one 4-bit qmv, x [1, 4096], W [4096, 4096] g64. A CUDA graph of 256
    back-to-back calls over 32 weight copies (302 MB, larger than L2), timed with
    CUDA events; plus the same calls through b2q.quantized_matmul from pinned host
    memory (e2e)."""
    import torch

    import b2q
    from b2q import synth
    from b2q._lib import check, lib

    L = lib()
    sp = stream.cuda_stream
    copies = [synth.packed_weights((4096,), 4096, GS, device=dev, seed=500 + i) for i in range(C0_COPIES)]
    xs = synth.activations((C0_CALLS, 4096), device=dev, seed=501)
    y = torch.empty((C0_CALLS, 4096), dtype=torch.bfloat16, device=dev)
    ptrs = [(w.data_ptr(), s_.data_ptr(), b.data_ptr()) for (w, s_, b) in copies]

    def call(i):
        w, s_, b = ptrs[i % C0_COPIES]
        rc = L.b2q_qmm(xs[i].data_ptr(), w, s_, b, y[i].data_ptr(), 1, 4096, 4096, GS, 4, 1, sp)
        if rc:
            check(rc)

    with torch.cuda.stream(stream):
        for i in range(8):
            call(i)
    torch.cuda.synchronize(dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for i in range(C0_CALLS):
            call(i)
    with torch.cuda.stream(stream):
        g.replay()
    torch.cuda.synchronize(dev)
    reps = 8
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    with torch.cuda.stream(stream):
        for _ in range(reps):
            g.replay()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    us = e0.elapsed_time(e1) * 1000.0 / (reps * C0_CALLS)
    gbs = C0_BYTES / (us * 1e-6) / 1e9
    # e2e: through the public op, x copied in from pinned host memory and y read back per call
    hx = torch.empty((64, 1, 4096), dtype=torch.bfloat16).pin_memory()
    hx.copy_(xs[:64].view(64, 1, 4096).cpu())
    hy = torch.empty((1, 4096), dtype=torch.bfloat16).pin_memory()
    dx = torch.empty((1, 4096), dtype=torch.bfloat16, device=dev)
    with torch.cuda.stream(stream):
        for i in range(8):
            dx.copy_(hx[i], non_blocking=True)
            hy.copy_(b2q.quantized_matmul(dx, *copies[i % C0_COPIES]), non_blocking=True)
        torch.cuda.synchronize(dev)
        n = 512
        e0.record(stream)
        for i in range(n):
            dx.copy_(hx[i % 64], non_blocking=True)
            hy.copy_(b2q.quantized_matmul(dx, *copies[i % C0_COPIES]), non_blocking=True)
        e1.record(stream)
        torch.cuda.synchronize(dev)
    e2e_us = e0.elapsed_time(e1) * 1000.0 / n
    del g, copies
    torch.cuda.empty_cache()
    return {"workload": "config 0: qmv x [1,4096] . W[4096,4096]^T, 4-bit g64",
            "us_per_call": us, "calls_per_s": 1e6 / us,
            "form": f"CUDA graph of {C0_CALLS} calls over {C0_COPIES} weight copies "
                    f"({C0_COPIES * C0_BYTES / 1e6:.0f} MB, cold in L2)",
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm_peak, "unit": "GB/s", "frac": gbs / hbm_peak,
                         "peak_kind": peak_kind, "bytes_per_launch": C0_BYTES},
            "e2e": {"value": 1e6 / e2e_us, "unit": "calls/s", "us_per_call": e2e_us, "h2d_bytes_per_step": 8192,
                    "d2h_bytes_per_step": 8192, "api": "b2q.quantized_matmul (pinned host x in, y back each call)"}}


def _graph_us(stream, dev, n_calls, call, reps=8):
    """us per call of a CUDA graph of n_calls calls, replayed reps times."""
    import torch

    with torch.cuda.stream(stream):
        for i in range(min(8, n_calls)):
            call(i)
    torch.cuda.synchronize(dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for i in range(n_calls):
            call(i)
    with torch.cuda.stream(stream):
        g.replay()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    with torch.cuda.stream(stream):
        for _ in range(reps):
            g.replay()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    del g
    return e0.elapsed_time(e1) * 1000.0 / (reps * n_calls)


def run_lut(dev, stream, hbm_peak, peak_kind):
    """The metadata pair index of a tensor (TrackAffineLUT): one-row products with each
    group's scale / bias read through a load-time table (u16 index per group in
    place of two bf16), against the plain product on the same weights. Config
    0's shape (graph of 256 calls over 32 copies) and an lm_head-sized product
    (N = 151,936; graph of 16 calls over 2 copies). The weights' metadata is the
    configs' own distribution, whose distinct pairs fit the table."""
    import torch

    from b2q import lut, synth
    from b2q._lib import check, lib

    L = lib()
    sp = stream.cuda_stream
    out = {}
    for name, N, copies_n, calls in (("c0", 4096, C0_COPIES, C0_CALLS), ("lm_head", 151936, 2, 16)):
        K = 4096
        copies = [synth.packed_weights((N,), K, GS, device=dev, seed=700 + i) for i in range(copies_n)]
        metas = [lut.AffineLUT.build(s_, b) for (_, s_, b) in copies]
        if any(m is None for m in metas):
            out[name] = {"skipped": "metadata not indexable"}
            continue
        xs = synth.activations((calls, K), device=dev, seed=701)
        y = torch.empty((calls, N), dtype=torch.bfloat16, device=dev)

        def plain(i):
            w, s_, b = copies[i % copies_n]
            rc = L.b2q_qmm(xs[i].data_ptr(), w.data_ptr(), s_.data_ptr(), b.data_ptr(), y[i].data_ptr(), 1, N, K, GS,
                           4, 1, sp)
            if rc:
                check(rc)

        def through_table(i):
            w = copies[i % copies_n][0]
            m = metas[i % copies_n]
            rc = L.b2q_qmv_lut(xs[i].data_ptr(), w.data_ptr(), m.index.data_ptr(), m.table.data_ptr(), m.count,
                               y[i].data_ptr(), N, K, GS, 4, sp)
            if rc:
                check(rc)

        us_plain = _graph_us(stream, dev, calls, plain)
        us_lut = _graph_us(stream, dev, calls, through_table)
        b_plain = N * (K // 2 + 4 * K // GS) + 2 * K + 2 * N
        count = max(m.count for m in metas)
        b_lut = N * (K // 2 + 2 * K // GS) + count * 4 + 2 * K + 2 * N
        out[name] = {"N": N, "K": K, "table_entries": count,
                     "us_per_call": us_lut, "us_per_call_plain": us_plain,
                     "bytes_per_call": b_lut, "bytes_per_call_plain": b_plain,
                     "roofline": {"bound": "hbm", "achieved": b_lut / (us_lut * 1e-6) / 1e9, "peak": hbm_peak,
                                  "unit": "GB/s", "frac": b_lut / (us_lut * 1e-6) / 1e9 / hbm_peak,
                                  "peak_kind": peak_kind},
                     "form": f"CUDA graph of {calls} calls over {copies_n} weight copies"}
        del copies, metas, xs, y
        torch.cuda.empty_cache()
    return out


EP_PROMPT, EP_NEW = 8192, 512


def run_ep_decoder(dev, world, rank, comm, pg, hbm_peak, peak_kind, n_new=EP_NEW, n_layers=48):
    """Config 4: the config-3 model with every MoE layer's experts sharded over the
    ranks (attention replicated); prefill 8192 random ids, then greedy tokens, each
    one replay of the captured step (NCCL all-reduce per layer inside the graph).
    Times are the max over ranks."""
    import torch

    from b2q.model import Decoder, DecoderConfig

    cfg = DecoderConfig(max_seq=EP_PROMPT + n_new, n_layers=n_layers, mtp=False)
    dec = Decoder(cfg, device=dev, seed=11, expert_parallel=(comm, world, rank))
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    prompt = torch.randint(0, cfg.vocab, (EP_PROMPT,), generator=g, device=dev, dtype=torch.int32)
    replay, tok, pos, lg = dec.decode_graph()
    dec.forward(prompt, 0)  # warm-up prefill
    torch.cuda.synchronize(dev)

    def max_over_ranks(ms):
        if pg is None:
            return ms
        t = torch.tensor([ms], device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        return float(t.item())

    if pg is not None:
        pg.barrier()
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p0.record()
    _, logits = dec.forward(prompt, 0)
    p1.record()
    torch.cuda.synchronize(dev)
    prefill_ms = max_over_ranks(p0.elapsed_time(p1))
    tok.copy_(logits.argmax(-1).to(torch.int32).view(1))
    pos.fill_(EP_PROMPT)
    torch.cuda.synchronize(dev)
    if pg is not None:
        pg.barrier()
    d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    d0.record()
    for _ in range(1, n_new):
        replay()
    d1.record()
    torch.cuda.synchronize(dev)
    ms_tok = max_over_ranks(d0.elapsed_time(d1) / (n_new - 1))
    status = dec.status()
    del replay, dec
    torch.cuda.empty_cache()
    return {"workload": f"config 4: the config-3 model ({n_layers} layers) expert-parallel over {world} GPU(s), "
                        f"experts {cfg.n_experts}/{world} per GPU, attention replicated; prompt {EP_PROMPT} random "
                        f"ids then {n_new} greedy tokens",
            "decode_tok_s": 1000.0 / ms_tok, "ms_per_token": ms_tok, "prefill_tok_s": EP_PROMPT * 1000.0 / prefill_ms,
            "prefill_ms": prefill_ms, "device_status": status,
            "decode_form": "one CUDA-graph replay per token; one NCCL all-reduce of the fp32 hidden partial per "
                           "layer inside the graph; prefill MoE layers through the all-reduce form"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=60000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", default="b2q", choices=["b2q", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--layers", type=int, default=N_LAYERS, help="rotating layers (cold-L2 decode)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-decoder", action="store_true", help="skip the config-3 full-decoder leg")
    ap.add_argument("--no-c0", action="store_true", help="skip the config-0 single-qmv leg")
    ap.add_argument("--ep-nccl", action="store_true",
                    help="expert parallel: one-token layers end in an NCCL all-reduce instead of the default "
                         "reduction over peer memory inside the kernel (b2q_ep_peer_setup / _open)")
    ap.add_argument("--decoder-only", type=int, default=0, metavar="TOKENS",
                    help="run only the config-3 leg with this many generated tokens (a short case for profiling)")
    ap.add_argument("--decoder-layers", type=int, default=48, help="layers of the config-3 model (48 in the spec)")
    ap.add_argument("--ep-decoder", type=int, default=0, metavar="TOKENS",
                    help="run only the config-4 leg (expert-parallel full model over the launched ranks)")
    args = ap.parse_args()
    args.ep_peer = not args.ep_nccl
    args.warmup = max(3, args.warmup)

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        run_reference(args, rank, world)
        return

    import torch

    import b2q
    from b2q import synth
    from b2q._lib import check, lib

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if args.decoder_only:
        hbm_peak, _, peak_kind = load_peaks()
        d = run_decoder(dev, hbm_peak, peak_kind, n_new=max(2, args.decoder_only), prefill_warmup=1,
                        n_layers=args.decoder_layers)
        print(json.dumps({"metric": "config 3 decode tok/s (bs=1)", "value": d.get("decode_tok_s"), "unit": "tok/s",
                          "n_gpus": 1, "decoder": d}), flush=True)
        return
    pg = None
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta

        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
        pg = dist

    hbm_peak, tc_peak, peak_kind = load_peaks()
    L = lib()
    if args.ep_decoder:
        from b2q.ep import EPComm

        comm4 = EPComm(world, rank, group=pg.group.WORLD) if world > 1 else None
        d = run_ep_decoder(dev, world, rank, comm4, pg, hbm_peak, peak_kind, n_new=max(2, args.ep_decoder),
                           n_layers=args.decoder_layers)
        if comm4 is not None:
            torch.cuda.synchronize(dev)
            comm4.close()
        if rank == 0:
            print(json.dumps({"metric": "config 4 decode tok/s (bs=1)", "value": d["decode_tok_s"], "unit": "tok/s",
                              "n_gpus": world, "decoder": d}), flush=True)
        if pg:
            pg.destroy_process_group()
        return

    # ---------------- decode (config 1) ----------------
    n_layers = max(1, args.layers)
    layers = [synth.moe_layer(E, H, F, GS, device=dev, seed=100 + 7 * i) for i in range(n_layers)]
    routers = [synth.router_weight(E, H, device=dev, seed=200 + i) for i in range(n_layers)]
    xs = synth.activations((N_TOKENS, H), device=dev, seed=1)
    out = torch.empty((1, H), dtype=torch.bfloat16, device=dev)
    ws_bytes = L.b2q_moe_decode_workspace_size(1, H, E, F, TOPK)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=dev)
    stream = torch.cuda.Stream(device=dev)
    sp = stream.cuda_stream
    fn = L.b2q_moe_decode
    comm = None
    e_lo, e_local = 0, E
    if world > 1:
        # expert parallelism: this rank holds experts [e_lo, e_lo + e_local) of every layer
        from b2q.ep import EPComm, expert_range, shard_layer

        e_lo, e_local = expert_range(E, world, rank)
        layers = [shard_layer(Ld, e_lo, e_local) for Ld in layers]
        torch.cuda.empty_cache()
        comm = EPComm(world, rank, group=pg.group.WORLD)
        if args.ep_peer:
            comm.enable_peer(H, group=pg.group.WORLD)
        ws_bytes = L.b2q_ep_moe_decode_workspace_size(1, H, E, F, TOPK)
        ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=dev)
        partial = torch.empty((1, H), dtype=torch.float32, device=dev)
    argsets = []
    for i in range(n_layers):
        Ld = layers[i]
        argsets.append([Ld[k].data_ptr() for k in ("wg", "sg", "bg", "wu", "su", "bu", "wd", "sd", "bd")])
    xbase, xstride = xs.data_ptr(), H * 2
    outp, wsp = out.data_ptr(), ws.data_ptr()

    if comm is None:
        def step(i):
            j = i % n_layers
            rc = fn(xbase + (i % N_TOKENS) * xstride, routers[j].data_ptr(), *argsets[j], outp, None, None, None,
                    1, H, E, F, TOPK, GS, 4, wsp, ws_bytes, sp)
            if rc:
                check(rc)
    else:
        epfn, commp, pp = L.b2q_ep_moe_decode, comm.ptr, partial.data_ptr()

        def step(i):
            j = i % n_layers
            rc = epfn(commp, xbase + (i % N_TOKENS) * xstride, routers[j].data_ptr(), *argsets[j], pp, outp, None,
                      None, 1, H, E, F, TOPK, e_lo, e_local, GS, 4, wsp, ws_bytes, sp)
            if rc:
                check(rc)

    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            step(i)
    torch.cuda.synchronize(dev)
    if pg:
        pg.barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    graphs = None
    if comm is None or args.ep_peer:
        # The K steps replay from CUDA graphs of G captured steps (step i reads token
        # i mod 4096 and layer i mod 8, as in the launch loop). The launch loop is
        # timed too and reported beside it. Expert parallel with the peer-memory
        # exchange: each step is one kernel launch, captured the same way. (With
        # the NCCL all-reduce the steps are timed as a launch loop: a capture of
        # the steps' NCCL calls in this leg did not complete on two GPUs.)
        ev0.record(stream)
        for i in range(args.steps):
            step(args.warmup + i)
        ev1.record(stream)
        torch.cuda.synchronize(dev)
        loop_ms = ev0.elapsed_time(ev1) / args.steps
        G = min(args.steps, 240)
        reps, rem = divmod(args.steps, G)

        def capture(first, count):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                for i in range(count):
                    step(first + i)
            return g

        graphs = [capture(args.warmup, G)] * reps
        if rem:
            graphs.append(capture(args.warmup + reps * G, rem))
        with torch.cuda.stream(stream):
            graphs[0].replay()  # untimed warm replay
        torch.cuda.synchronize(dev)
        if pg:
            pg.barrier()
    with ClockSampler(local_rank) as clk:
        torch.cuda.synchronize(dev)
        if pg:
            # the ranks enter the timed region together: starting the clock
            # sampler takes each rank a different time, and with expert
            # parallelism every step waits for every rank
            pg.barrier()
        if graphs is not None:
            with torch.cuda.stream(stream):
                # a spin kernel keeps the stream busy while the host enqueues the
                # start event and the graph launches, so the timed region holds
                # the K steps and not the host's launch of the first graph
                torch.cuda._sleep(200_000)
                ev0.record(stream)
                for g in graphs:
                    g.replay()
                ev1.record(stream)
        else:
            ev0.record(stream)
            for i in range(args.steps):
                step(args.warmup + i)
            ev1.record(stream)
        torch.cuda.synchronize(dev)
    ms_total = ev0.elapsed_time(ev1)
    graph_timed = graphs is not None
    graphs = None
    if pg:
        t = torch.tensor([ms_total], device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        ms_total = float(t.item())
    st = L.b2q_workspace_status(wsp, ws_bytes, sp) if comm is None else 0
    if st != 0:
        raise RuntimeError(f"device-side error {st} during the timed decode loop")
    ms_step = ms_total / args.steps
    tok_s = 1000.0 / ms_step  # one token per step for the whole job
    achieved = DECODE_BYTES / (ms_step * 1e-3) / 1e9
    clocks = clk.summary()

    # ---------------- e2e through the public API ----------------
    if comm is None:
        moe = [b2q.MoE(routers[i], layers[i], TOPK, GS) for i in range(n_layers)]
    else:
        from b2q.ep import EPMoE

        moe = [EPMoE(routers[i], layers[i], E, e_lo, TOPK, comm, GS) for i in range(n_layers)]
    n_e2e = 0 if args.no_e2e else min(args.steps, 3000)
    host_x = torch.empty((n_e2e + args.warmup, 1, H), dtype=torch.bfloat16).pin_memory()
    host_x.copy_(xs[: (n_e2e + args.warmup)].view(-1, 1, H).cpu())
    host_out = torch.empty((1, H), dtype=torch.bfloat16).pin_memory()
    dx = torch.empty((1, H), dtype=torch.bfloat16, device=dev)
    dy = torch.empty((1, H), dtype=torch.bfloat16, device=dev)
    # the one-token call writes a persistent output buffer (no allocation per call)
    call_kw = {"out": dy} if comm is None else {}
    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            dx.copy_(host_x[i], non_blocking=True)
            y = moe[i % n_layers](dx, **call_kw)
            host_out.copy_(y, non_blocking=True)
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(n_e2e):
            dx.copy_(host_x[args.warmup + i], non_blocking=True)
            y = moe[i % n_layers](dx, **call_kw)
            host_out.copy_(y, non_blocking=True)
        e1.record(stream)
        torch.cuda.synchronize(dev)
    py_ms = e0.elapsed_time(e1) / max(1, n_e2e) if n_e2e else float("nan")
    e2e_ms = py_ms
    e2e_api = ("b2q.MoE.__call__" if comm is None else "b2q.ep.EPMoE.__call__") + \
        " (pinned host token in, pinned host output back each step)"
    if comm is None and n_e2e:
        # the C ABI from a native host loop (as the reference's Swift runner would
        # call it): b2q_moe_decode per step, token row in from pinned host memory and
        # output row back every step, copies double-buffered on a second stream
        import ctypes

        hx = torch.empty((N_TOKENS, H), dtype=torch.bfloat16).pin_memory()
        hx.copy_(xs.cpu())
        ho = torch.empty((H,), dtype=torch.bfloat16).pin_memory()
        dx2 = torch.empty((2, H), dtype=torch.bfloat16, device=dev)
        dy2 = torch.empty((2, H), dtype=torch.bfloat16, device=dev)
        wr_arr = (ctypes.c_void_p * n_layers)(*[routers[j].data_ptr() for j in range(n_layers)])
        w9_arr = (ctypes.c_void_p * (9 * n_layers))(*[q for j in range(n_layers) for q in argsets[j]])
        ms = ctypes.c_float(0.0)
        check(L.b2q_moe_decode_host_loop(hx.data_ptr(), N_TOKENS, ho.data_ptr(), wr_arr, w9_arr, n_layers, H, E, F,
                                         TOPK, GS, 4, dx2.data_ptr(), dy2.data_ptr(), wsp, ws_bytes, args.warmup,
                                         n_e2e, sp, ctypes.byref(ms)))
        e2e_ms = float(ms.value)
        e2e_api = ("b2q_moe_decode through the C ABI from a native host loop (b2q_moe_decode_host_loop): pinned "
                   "host token in and output back every step, copies double-buffered on a second stream")
    if pg:
        t = torch.tensor([e2e_ms], device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        e2e_ms = float(t.item())

    # ---------------- prefill (config 2) ----------------
    prefill = None
    if not args.no_prefill:
        del moe
        xp = synth.activations((PREFILL_T, H), device=dev, seed=3)
        pout = torch.empty((PREFILL_T, H), dtype=torch.bfloat16, device=dev)
        if comm is None:
            pws = b2q.Workspace(L.b2q_moe_prefill_workspace_size(PREFILL_T, H, E, F, TOPK), dev)

            def pstep(i):
                j = i % n_layers
                rc = L.b2q_moe_prefill(xp.data_ptr(), routers[j].data_ptr(), *argsets[j], pout.data_ptr(), None,
                                       None, PREFILL_T, H, E, F, TOPK, GS, 4, pws.ptr(), pws.buf.numel(), sp)
                if rc:
                    check(rc)
        else:
            pws = b2q.Workspace(L.b2q_ep_moe_prefill_workspace_size(PREFILL_T, H, E, F, TOPK), dev)
            ppart = torch.empty((PREFILL_T, H), dtype=torch.float32, device=dev)

            def pstep(i):
                j = i % n_layers
                rc = L.b2q_ep_moe_prefill(comm.ptr, xp.data_ptr(), routers[j].data_ptr(), *argsets[j],
                                          ppart.data_ptr(), pout.data_ptr(), None, None, PREFILL_T, H, E, F, TOPK,
                                          e_lo, e_local, GS, 4, pws.ptr(), pws.buf.numel(), sp)
                if rc:
                    check(rc)

        with torch.cuda.stream(stream):
            for i in range(3):
                pstep(i)
        torch.cuda.synchronize(dev)
        psteps = 10
        if pg:
            pg.barrier()
        p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        p0.record(stream)
        for i in range(psteps):
            pstep(i)
        p1.record(stream)
        torch.cuda.synchronize(dev)
        pms = p0.elapsed_time(p1) / psteps
        if pg:
            t = torch.tensor([pms], device=dev)
            pg.all_reduce(t, op=pg.ReduceOp.MAX)
            pms = float(t.item())
        tflops = PREFILL_FLOP / (pms * 1e-3) / 1e12
        a2a = None
        if comm is not None:
            # the all-to-all form: each rank owns a block of the 2048 tokens, rows travel to the
            # ranks holding their experts and the weighted partial rows travel back
            from b2q.ep import token_range

            t_lo, t_n = token_range(PREFILL_T, world, rank)
            t_max = max(token_range(PREFILL_T, world, r)[1] for r in range(world))
            aws = b2q.Workspace(L.b2q_ep_moe_prefill_a2a_workspace_size(t_max, H, E, F, TOPK, world), dev)
            xa = xp[t_lo:t_lo + t_n]

            def astep(i):
                j = i % n_layers
                rc = L.b2q_ep_moe_prefill_a2a(comm.ptr, xa.data_ptr(), routers[j].data_ptr(), *argsets[j],
                                              pout.data_ptr(), None, None, t_n, t_max, H, E, F, TOPK, GS, 4,
                                              aws.ptr(), aws.buf.numel(), sp)
                if rc:
                    check(rc)

            with torch.cuda.stream(stream):
                for i in range(3):
                    astep(i)
            torch.cuda.synchronize(dev)
            pg.barrier()
            a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a0.record(stream)
            for i in range(psteps):
                astep(i)
            a1.record(stream)
            torch.cuda.synchronize(dev)
            ams = a0.elapsed_time(a1) / psteps
            t = torch.tensor([ams], device=dev)
            pg.all_reduce(t, op=pg.ReduceOp.MAX)
            ams = float(t.item())
            a2a = {"ms_per_layer": ams, "tok_s": PREFILL_T * 1000.0 / ams,
                   "form": f"all-to-all: {t_max} tokens per rank at most, token rows dispatched once per "
                           "destination rank (NCCL grouped send/recv), fp32 partial rows returned and summed by "
                           "the owner; the counts are read on the host every call"}
        prefill = {"workload": "config 2: MoE layer prefill, 2048 tokens", "tok_s": PREFILL_T * 1000.0 / pms,
                   "all_to_all": a2a,
                   "ms_per_layer": pms, "roofline": {"bound": "tensor", "achieved": tflops, "peak": tc_peak,
                                                     "unit": "TFLOP/s", "frac": tflops / tc_peak,
                                                     "peak_kind": peak_kind,
                                                     "traffic": load_traffic("moe_prefill_c2.json")}}

    # ---------------- single qmv (config 0), one GPU ----------------
    c0 = None
    if world == 1 and not args.no_c0:
        c0 = run_c0(dev, stream, hbm_peak, peak_kind)
    affine_lut = None
    if world == 1 and not args.no_c0:
        affine_lut = run_lut(dev, stream, hbm_peak, peak_kind)

    # ---------------- full decoder (config 3), one GPU ----------------
    decoder = None
    if not args.no_decoder and world == 1:
        decoder = run_decoder(dev, hbm_peak, peak_kind)

    if comm is not None:
        torch.cuda.synchronize(dev)
        comm.close()
    if rank != 0:
        if pg:
            pg.destroy_process_group()
        return
    cpu = None
    if not args.no_cpu_baseline and world == 1:
        cpu = cpu_baseline_sample()
        if prefill is not None:
            prefill["cpu_baseline"] = prefill_cpu_baseline(cpu["row_s"], cpu["kind"])
        if decoder is not None and "decode_tok_s" in decoder:
            decoder["cpu_baseline"] = decoder_cpu_baseline(cpu["row_s"], cpu["kind"])
        if c0 is not None:
            c0["cpu_baseline"] = {"value": 1.0 / (cpu["row_s"] * 4096), "unit": "calls/s", "cores": 1,
                                  "kind": cpu["kind"],
                                  "sample": "measured per-row time of the reference's MLX CPU kernel (K=4096 4-bit "
                                            "g64, bf16 sum) x 4096 rows"}
    line = {
        "metric": METRIC,
        "value": tok_s,
        "unit": "tok/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_step,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded; random-init 4-bit experts)",
        "config": {"workload": WORKLOAD,
                   "parallelism": "single GPU" if world == 1 else
                   (f"ep{world}: experts sharded {E}/{world} per GPU, router replicated, the fp32 partials "
                    f"exchanged over peer memory inside the kernel (no collective call)" if args.ep_peer else
                    f"ep{world}: experts sharded {E}/{world} per GPU, router replicated, one NCCL all-reduce of "
                    f"the fp32 hidden vector per layer"),
                   "l2": f"cold: {n_layers} rotating layers ({n_layers * E * EXPERT_BYTES / 1e9:.1f} GB experts) "
                         f"and a fresh token per step"},
        "decode_form": ("CUDA-graph replays of the captured steps, the stream kept busy while the first graph "
                        f"is launched (launch loop: {loop_ms * 1000.0:.2f} us per step)" if graph_timed
                        else "launch loop"),
        "gather_qmv_hbm_gbs": achieved,
        "hbm_frac_of_8tbs": achieved / 8000.0,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                     "frac": achieved / hbm_peak, "peak_kind": peak_kind,
                     "bytes_per_launch": DECODE_BYTES,
                     "traffic": load_traffic("moe_decode_c1.json")},
        "e2e": ({"value": 1000.0 / e2e_ms, "unit": "tok/s", "h2d_bytes_per_step": H * 2, "d2h_bytes_per_step": H * 2,
                 "steps": n_e2e, "api": e2e_api,
                 "python_api": {"value": 1000.0 / py_ms, "unit": "tok/s",
                                "api": ("b2q.MoE.__call__" if comm is None else "b2q.ep.EPMoE.__call__")
                                + " from a Python loop (pinned host token in, output back each step)"}}
                if n_e2e else None),
        # one kernel per step (one GPU, or the peer-memory exchange); with the NCCL
        # all-reduce: the kernel, the NCCL kernel and the bf16 conversion
        "gpu_launches": args.steps * (1 if world == 1 or args.ep_peer else 3),
        "clocks": clocks,
        "prefill": prefill,
        "decoder": decoder,
        "c0": c0,
        "affine_lut": affine_lut,
        "cpu_baseline": cpu,
    }
    print(json.dumps(line), flush=True)
    if pg:
        pg.destroy_process_group()


if __name__ == "__main__":
    main()
