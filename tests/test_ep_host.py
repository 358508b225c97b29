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


def test_expert_range_matches_the_library_rule(b2q_mod):
    """The Python rule, the C-ABI rule (b2q_ep_expert_range, host arithmetic only)
    and the oracle's owner function agree, so the dispatch routes to the rank that
    holds the expert."""
    import ctypes

    from b2q.ep import expert_range, token_range
    from oracle.oracle import ep_owner

    lib = b2q_mod.lib()
    for E in (16, 128, 13, 8):
        for world in range(1, 9):
            if world > E:
                continue
            for r in range(world):
                lo, n = ctypes.c_int(), ctypes.c_int()
                assert lib.b2q_ep_expert_range(E, world, r, ctypes.byref(lo), ctypes.byref(n)) == 0
                assert (lo.value, n.value) == expert_range(E, world, r)
                assert all(ep_owner(e, E, world) == r for e in range(lo.value, lo.value + n.value))
    lo, n = ctypes.c_int(), ctypes.c_int()
    assert lib.b2q_ep_expert_range(4, 8, 0, ctypes.byref(lo), ctypes.byref(n)) == -1
    for T, world in ((96, 2), (7, 3), (0, 2), (5, 8)):
        blocks = [token_range(T, world, r) for r in range(world)]
        assert sum(n for _, n in blocks) == T
        assert [lo for lo, _ in blocks] == [sum(n for _, n in blocks[:r]) for r in range(world)]


def test_a2a_plan_dedups_per_rank():
    from oracle.oracle import ep_a2a_plan

    idx = np.array([[0, 1, 8], [9, 10, 15], [2, 3, 4], [0, 15, 7]], np.uint32)
    pos, counts = ep_a2a_plan(idx, 16, 2)
    assert counts.tolist() == [3, 3]
    assert pos.tolist() == [[0, 0], [-1, 1], [1, -1], [2, 2]]


def test_a2a_argument_checks(b2q_mod):
    lib = b2q_mod.lib()
    # more ranks than the exchange supports, or than experts: refused on the host
    assert lib.b2q_ep_a2a_dispatch(*([None] * 8), 4, 256, 16, 2, 9, None, 0, None) == -1
    assert lib.b2q_ep_a2a_dispatch_workspace_size(4, 256, 4, 2, 8) == 0
    assert lib.b2q_ep_moe_prefill_a2a_workspace_size(64, 1024, 16, 512, 4, 9) == 0
    assert lib.b2q_ep_moe_prefill_a2a_workspace_size(64, 1024, 16, 512, 4, 2) > 2 * 64 * 1024 * (2 + 2 + 4 + 4)
    # T above T_max, and shapes the tensor cores do not take
    assert lib.b2q_ep_moe_prefill_a2a(*([None] * 15), 65, 64, 1024, 16, 512, 4, 64, 4, None, 0, None) == -1
    assert lib.b2q_ep_moe_prefill_a2a(*([None] * 15), 8, 64, 1000, 16, 512, 4, 64, 4, None, 0, None) in (-1, -2)
    assert lib.b2q_ep_a2a_combine(None, None, None, 4, 1026, 2, None) == -1
    assert lib.b2q_ep_a2a_combine(None, None, None, 0, 1024, 2, None) == 0


def _a2a_rank_main(rank, world, port, T, result_path):
    """The all-to-all protocol over gloo with the oracle as the products: own
    tokens -> plan -> rows and (expert, weight) pairs to their ranks -> local
    partial rows -> back to the owner -> sum in rank order."""
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from b2q.ep import expert_range, token_range
        from oracle.oracle import ep_a2a_plan

        o, x, layer, idx, w, shp = _problem(S=T)
        k, H = shp["k"], shp["H"]
        t_lo, t_n = token_range(T, world, rank)
        my_idx, my_w = idx[t_lo:t_lo + t_n], w[t_lo:t_lo + t_n]
        pos, counts = ep_a2a_plan(my_idx, shp["E"], world)
        # counts to everyone (the library all-gathers them)
        allc = torch.zeros(world * world, dtype=torch.int32)
        dist.all_gather(list(allc.view(world, world).unbind(0)), torch.from_numpy(counts))
        cm = allc.view(world, world).numpy()
        blocks = []
        for d in range(world):
            rows = [t for t in range(t_n) if pos[t, d] >= 0]
            blocks.append((x[t_lo + np.array(rows, int)].reshape(-1, H) if rows else np.zeros((0, H), np.uint16),
                           my_idx[rows].reshape(-1, k), my_w[rows].reshape(-1, k)))
        recv = []
        for s in range(world):
            n = int(cm[s, rank])
            if s == rank:
                recv.append(blocks[rank])
                continue
            xb = torch.zeros((n, H), dtype=torch.int16)
            ib = torch.zeros((n, k), dtype=torch.int64)
            wb = torch.zeros((n, k), dtype=torch.float32)
            # the lower rank of the pair sends first (gloo send blocks until received)
            for turn in sorted(((rank, s), (s, rank))):
                if turn[0] == rank and cm[rank, s]:
                    bx, bi, bw = blocks[s]
                    dist.send(torch.from_numpy(bx.view(np.int16).copy()), s)
                    dist.send(torch.from_numpy(bi.astype(np.int64)), s)
                    dist.send(torch.from_numpy(bw.astype(np.float32)), s)
                elif turn[0] == s and n:
                    dist.recv(xb, s)
                    dist.recv(ib, s)
                    dist.recv(wb, s)
            recv.append((xb.numpy().view(np.uint16), ib.numpy().astype(np.uint32), wb.numpy()))
        e_lo, e_local = expert_range(shp["E"], world, rank)
        parts = []
        for rx, ri, rw in recv:
            sh = dict(shp, S=rx.shape[0])
            parts.append(_partial(o, rx, layer, ri, rw, sh, e_lo, e_local) if rx.shape[0] else np.zeros((0, H), np.float32))
        # partial rows back to the owners; the owner sums in rank order
        ret = [None] * world
        for s in range(world):
            if s == rank:
                ret[rank] = parts[rank]
                continue
            buf = torch.zeros((int(cm[rank, s]), H), dtype=torch.float32)
            for turn in sorted(((rank, s), (s, rank))):
                if turn[0] == rank and cm[s, rank]:
                    dist.send(torch.from_numpy(np.ascontiguousarray(parts[s])), s)
                elif turn[0] == s and cm[rank, s]:
                    dist.recv(buf, s)
            ret[s] = buf.numpy()
        out = np.zeros((t_n, H), np.float32)
        for t in range(t_n):
            first = True
            for d in range(world):
                if pos[t, d] < 0:
                    continue
                v = ret[d][pos[t, d]]
                out[t] = v if first else (out[t] + v).astype(np.float32)
                first = False
        np.save(result_path + f".{rank}.npy", out)
    finally:
        dist.destroy_process_group()


def test_a2a_layer_on_two_gloo_ranks(tmp_path):
    import torch.multiprocessing as mp

    from oracle.oracle import bf16_to_f32

    T = 5
    path = str(tmp_path / "a2a")
    mp.start_processes(_a2a_rank_main, args=(2, _free_port(), T, path), nprocs=2, start_method="spawn", join=True)
    got = np.concatenate([np.load(path + f".{r}.npy") for r in range(2)])
    o, x, layer, idx, w, shp = _problem(S=T)
    full = o.moe_experts_decode(x, idx, w, layer, shp["k"], group_size=shp["gs"])
    e = rel_l2(got, bf16_to_f32(full))
    assert e < REL_L2, e


class _RecordingLib:
    """Stands in for the library in the handshake test: records what the
    host side hands to each entry point (no device, no NCCL)."""

    def __init__(self, rank, world):
        import ctypes

        self.ctypes, self.rank, self.world = ctypes, rank, world
        self.uid_seen = self.opened = None
        self.setup_H = None

    def b2q_ep_unique_id(self, p, n):
        self.ctypes.memmove(p, bytes((i * 7 + 3) % 256 for i in range(n)), n)
        return 0

    def b2q_ep_comm_init(self, pptr, world, rank, uid, n):
        assert (world, rank) == (self.world, self.rank)
        self.uid_seen = self.ctypes.string_at(uid, n)
        return 0

    def b2q_ep_peer_setup(self, comm, H, h, hb):
        self.setup_H = H
        self.ctypes.memmove(h, bytes([0x40 + self.rank]) * hb, hb)
        return 0

    def b2q_ep_peer_open(self, comm, handles, hb):
        self.opened = self.ctypes.string_at(handles, hb * self.world)
        return 0


def _handshake_rank_main(rank, world, port, result_path):
    import json

    import torch.distributed as dist

    import b2q.ep as ep

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        fake = _RecordingLib(rank, world)
        ep.lib = lambda: fake
        comm = ep.EPComm(world, rank, group=dist.group.WORLD)
        comm.enable_peer(4096, group=dist.group.WORLD)
        with open(f"{result_path}.{rank}", "w") as f:
            json.dump({"uid": fake.uid_seen.hex(), "opened": fake.opened.hex(), "H": fake.setup_H}, f)
    finally:
        dist.destroy_process_group()


def test_comm_handshakes_on_gloo_ranks(tmp_path):
    """EPComm over a gloo group: every rank's communicator gets rank 0's NCCL
    id, and enable_peer hands b2q_ep_peer_open every rank's exchange handle in
    rank order (the layout the library indexes by rank)."""
    import json

    import torch.multiprocessing as mp

    world = 3
    path = str(tmp_path / "hs")
    mp.start_processes(_handshake_rank_main, args=(world, _free_port(), path), nprocs=world, start_method="spawn",
                       join=True)
    uid = bytes((i * 7 + 3) % 256 for i in range(128)).hex()
    want = b"".join(bytes([0x40 + r]) * 64 for r in range(world)).hex()
    for r in range(world):
        with open(f"{path}.{r}") as f:
            got = json.load(f)
        assert got == {"uid": uid, "opened": want, "H": 4096}
