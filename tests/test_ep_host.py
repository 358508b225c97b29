"""Expert-parallel host logic on CPU: expert ranges, and the sharded layer on
two gloo ranks (each rank's partial from the oracle over its own experts,
summed by all_reduce) against the single-rank oracle layer."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

from conftest import REL_L2, rel_l2


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def test_expert_ranges_partition_the_experts():
    from b2q.ep import expert_range

    for E, world in ((128, 1), (128, 2), (128, 8), (10, 3), (7, 7)):
        covered = []
        for r in range(world):
            lo, n = expert_range(E, world, r)
            assert n >= 1
            covered.extend(range(lo, lo + n))
        assert covered == list(range(E))
    with pytest.raises(ValueError):
        expert_range(4, 8, 0)


def _problem(seed=0, S=2, H=256, E=8, F=128, k=3, gs=64):
    rng = np.random.default_rng(seed)
    from oracle.oracle import Oracle, f32_to_bf16

    o = Oracle()

    def packed(rows, K):
        w = rng.integers(0, 2**32, size=(rows, K // 8), dtype=np.uint32)
        s = f32_to_bf16(rng.uniform(0.002, 0.02, size=(rows, K // gs)).astype(np.float32))
        from oracle.oracle import bf16_to_f32
        b = f32_to_bf16((-8.0 * bf16_to_f32(s) + rng.normal(0, 1e-3, size=s.shape)).astype(np.float32))
        return w, s, b

    layer = {}
    for nm, (rows, K) in (("g", (F, H)), ("u", (F, H)), ("d", (H, F))):
        ws, ss, bs = zip(*[packed(rows, K) for _ in range(E)])
        layer["w" + nm], layer["s" + nm], layer["b" + nm] = np.stack(ws), np.stack(ss), np.stack(bs)
    x = f32_to_bf16(rng.normal(size=(S, H)).astype(np.float32))
    wr = f32_to_bf16((0.02 * rng.normal(size=(E, H))).astype(np.float32))
    logits = o.router_logits(x, wr)
    idx, w = o.route(logits, k)
    return o, x, layer, idx, w, dict(S=S, H=H, E=E, F=F, k=k, gs=gs)


def _partial(o, x, layer, idx, w, shp, e_lo, e_local):
    """fp32 partial of the experts [e_lo, e_lo + e_local): colsum association
    over all k slots with zeros for the slots held elsewhere."""
    from oracle.oracle import bf16_to_f32, f32_to_bf16

    S, H, k, gs = shp["S"], shp["H"], shp["k"], shp["gs"]
    out = np.zeros((S, H), np.float32)
    for t in range(S):
        prod = np.zeros((k, H), np.float32)
        for j in range(k):
            e = int(idx[t, j])
            if not (e_lo <= e < e_lo + e_local):
                continue
            g = o.qmv_metal_f32(x[t:t + 1], layer["wg"][e], layer["sg"][e], layer["bg"][e], gs)
            u = o.qmv_metal_f32(x[t:t + 1], layer["wu"][e], layer["su"][e], layer["bu"][e], gs)
            act = o.swiglu(f32_to_bf16(g), f32_to_bf16(u)).reshape(1, -1)
            y = o.qmv_metal_f32(act, layer["wd"][e], layer["sd"][e], layer["bd"][e], gs)
            prod[j] = bf16_to_f32(f32_to_bf16(y)).reshape(-1) * np.float32(w[t, j])
        TY = min(k, 8)
        tt = [np.zeros(H, np.float32) for _ in range(TY)]
        for q in range(TY):
            a = np.zeros(H, np.float32)
            for r in range(q, k, TY):
                a = (prod[r] + a).astype(np.float32)
            tt[q] = a
        total = tt[0]
        for q in range(1, TY):
            total = (tt[q] + total).astype(np.float32)
        out[t] = total
    return out


def _rank_main(rank, world, port, result_path):
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from b2q.ep import expert_range

        o, x, layer, idx, w, shp = _problem()
        e_lo, e_local = expert_range(shp["E"], world, rank)
        part = torch.from_numpy(_partial(o, x, layer, idx, w, shp, e_lo, e_local))
        dist.all_reduce(part)
        if rank == 0:
            np.save(result_path, part.numpy())
    finally:
        dist.destroy_process_group()


def test_sharded_layer_on_two_gloo_ranks(tmp_path):
    import torch.multiprocessing as mp

    from oracle.oracle import bf16_to_f32

    path = str(tmp_path / "sum.npy")
    mp.start_processes(_rank_main, args=(2, _free_port(), path), nprocs=2, start_method="spawn", join=True)
    summed = np.load(path)
    o, x, layer, idx, w, shp = _problem()
    full = o.moe_experts_decode(x, idx, w, layer, shp["k"], group_size=shp["gs"])
    e = rel_l2(summed, bf16_to_f32(full))
    assert e < REL_L2, e
    # one rank holding every expert is the single-GPU association exactly
    one = _partial(o, x, layer, idx, w, shp, 0, shp["E"])
    from oracle.oracle import f32_to_bf16

    assert np.array_equal(f32_to_bf16(one), full)
