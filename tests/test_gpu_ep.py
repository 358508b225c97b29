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
