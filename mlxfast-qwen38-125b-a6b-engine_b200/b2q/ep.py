"""Expert parallelism: experts sharded over the ranks of a process group.

The reference's MoE layer with its experts sharded over ranks; every rank
holds the router and a contiguous block of experts. Two forms:

* all-reduce (`EPMoE.__call__`): tokens replicated; every rank computes the
  routing in full, multiplies the selected experts it holds and sums its
  weighted outputs into an fp32 partial; one all-reduce of the partial per
  layer gives the layer output (NCCL, inside the library, on the caller's
  stream). Decode and prefill.
* all-to-all (`EPMoE.prefill_a2a`): each rank owns its own tokens; a token row
  travels once to every rank holding one of its experts (dispatch), the
  weighted partial rows travel back (combine). Prefill. The phases are also
  callable one by one (`a2a_dispatch`, `a2a_experts`, `a2a_combine`) for a
  runtime that moves the blocks through its own transport.

Host-side pieces here are plain Python (expert ranges, shard slicing, the NCCL
id handshake through torch.distributed); the products run through the
library's b2q_ep_* entry points.
"""
from __future__ import annotations

import ctypes

import torch

from ._lib import check, lib

NCCL_ID_BYTES = 128


def expert_range(E: int, world: int, rank: int) -> tuple[int, int]:
    """(e_lo, e_local) of `rank`: contiguous blocks, the first E % world ranks one larger
    (the rule of b2q_ep_expert_range, which the all-to-all dispatch routes by)."""
    if not (0 <= rank < world) or E < world:
        raise ValueError(f"cannot shard {E} experts over {world} ranks")
    base, extra = divmod(E, world)
    e_lo = rank * base + min(rank, extra)
    return e_lo, base + (1 if rank < extra else 0)


def token_range(T: int, world: int, rank: int) -> tuple[int, int]:
    """(t_lo, t_local): the contiguous block of T replicated tokens a rank owns in the
    all-to-all form (the first T % world ranks one token more)."""
    if not (0 <= rank < world) or T < 0:
        raise ValueError(f"bad token split: T={T} world={world} rank={rank}")
    base, extra = divmod(T, world)
    return rank * base + min(rank, extra), base + (1 if rank < extra else 0)


def shard_layer(layer: dict, e_lo: int, e_local: int) -> dict:
    """The local experts' stacked tensors ([e_local, ...], contiguous)."""
    return {k: v[e_lo:e_lo + e_local].contiguous() for k, v in layer.items()}


class EPComm:
    """An NCCL communicator of the library over `world` ranks.

    With a torch.distributed group (any backend) the NCCL id is made on rank 0
    and broadcast through it; a single rank needs no communicator."""

    def __init__(self, world: int = 1, rank: int = 0, group=None):
        self.world, self.rank = world, rank
        self.ptr = ctypes.c_void_p()
        uid = (ctypes.c_char * NCCL_ID_BYTES)()
        if world > 1:
            import torch.distributed as dist

            buf = torch.zeros(NCCL_ID_BYTES, dtype=torch.uint8)
            if rank == 0:
                check(lib().b2q_ep_unique_id(ctypes.cast(uid, ctypes.c_void_p), NCCL_ID_BYTES))
                buf.copy_(torch.frombuffer(bytearray(bytes(uid)), dtype=torch.uint8))
            if group is not None and dist.get_backend(group) == "nccl":
                dev_buf = buf.cuda()
                dist.broadcast(dev_buf, 0, group=group)
                buf = dev_buf.cpu()
            else:
                dist.broadcast(buf, 0, group=group)
            ctypes.memmove(uid, bytes(buf.numpy().tobytes()), NCCL_ID_BYTES)
        check(lib().b2q_ep_comm_init(ctypes.byref(self.ptr), world, rank,
                                     ctypes.cast(uid, ctypes.c_void_p), NCCL_ID_BYTES))

    def enable_peer(self, H: int, group=None):
        """One-token layers of hidden size H reduce over peer memory from now on
        (b2q_ep_peer_setup / _open): every rank's exchange-buffer handle is
        gathered through the torch.distributed group. Every rank calls it."""
        if self.world < 2:
            return
        import torch.distributed as dist

        hb = 64
        h = (ctypes.c_char * hb)()
        check(lib().b2q_ep_peer_setup(self.ptr, H, ctypes.cast(h, ctypes.c_void_p), hb))
        mine = torch.frombuffer(bytearray(bytes(h)), dtype=torch.uint8)
        if group is not None and dist.get_backend(group) == "nccl":
            parts = [torch.empty(hb, dtype=torch.uint8, device="cuda") for _ in range(self.world)]
            dist.all_gather(parts, mine.cuda(), group=group)
            parts = [t.cpu() for t in parts]
        else:
            parts = [torch.empty(hb, dtype=torch.uint8) for _ in range(self.world)]
            dist.all_gather(parts, mine, group=group)
        allh = b"".join(bytes(t.numpy().tobytes()) for t in parts)
        buf = (ctypes.c_char * len(allh)).from_buffer_copy(allh)
        check(lib().b2q_ep_peer_open(self.ptr, ctypes.cast(buf, ctypes.c_void_p), hb))

    def close(self):
        if self.ptr:
            check(lib().b2q_ep_comm_destroy(self.ptr))
            self.ptr = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class EPMoE:
    """One MoE layer with this rank's experts [e_lo, e_lo + e_local) of E."""

    def __init__(self, router_weight, local_layer: dict, E: int, e_lo: int, k: int, comm: EPComm | None = None,
                 group_size: int = 64, bits: int = 4):
        self.wr, self.L = router_weight, local_layer
        self.E, self.e_lo, self.e_local = E, e_lo, local_layer["wg"].shape[0]
        self.k, self.gs, self.bits = k, group_size, bits
        self.comm = comm
        self._ws = {}

    def _workspace(self, kind, nbytes, device):
        w = self._ws.get(kind)
        if w is None or w.numel() < nbytes:
            w = torch.zeros(max(256, nbytes), dtype=torch.uint8, device=device)
            self._ws[kind] = w
        return w

    def __call__(self, x: torch.Tensor, return_partial: bool = False):
        T, H = x.shape
        F = self.L["wg"].shape[1]
        decode = T <= 8
        size_fn = lib().b2q_ep_moe_decode_workspace_size if decode else lib().b2q_ep_moe_prefill_workspace_size
        ws = self._workspace("decode" if decode else "prefill", size_fn(T, H, self.E, F, self.k), x.device)
        partial = torch.empty((T, H), dtype=torch.float32, device=x.device)
        out = torch.empty((T, H), dtype=torch.bfloat16, device=x.device)
        fn = lib().b2q_ep_moe_decode if decode else lib().b2q_ep_moe_prefill
        L = self.L
        check(fn(self.comm.ptr if self.comm else None, x.data_ptr(), self.wr.data_ptr(),
                 *[L[n].data_ptr() for n in ("wg", "sg", "bg", "wu", "su", "bu", "wd", "sd", "bd")],
                 partial.data_ptr(), out.data_ptr(), None, None, T, H, self.E, F, self.k, self.e_lo, self.e_local,
                 self.gs, self.bits, ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream))
        return (out, partial) if return_partial else out

    def prefill_a2a(self, x: torch.Tensor, T_max: int | None = None) -> torch.Tensor:
        """This rank's tokens x [T, H] through the all-to-all layer; returns their
        outputs [T, H] (bf16). Every rank of the communicator calls it (T may be 0);
        T_max must be at least every rank's T (it sizes the receive buffers)."""
        T, H = x.shape
        F = self.L["wg"].shape[1]
        world = self.comm.world if self.comm else 1
        rank = self.comm.rank if self.comm else 0
        lo, n = expert_range(self.E, world, rank)
        if (lo, n) != (self.e_lo, self.e_local):
            raise ValueError(f"rank {rank} holds experts [{self.e_lo}, {self.e_lo + self.e_local}), the all-to-all "
                             f"rule gives [{lo}, {lo + n})")
        T_max = max(1, T if T_max is None else T_max)
        size = lib().b2q_ep_moe_prefill_a2a_workspace_size(T_max, H, self.E, F, self.k, world)
        if size == 0:
            raise ValueError("ep prefill a2a: bad shape")
        ws = self._workspace("a2a", size, x.device)
        out = torch.empty((T, H), dtype=torch.bfloat16, device=x.device)
        L = self.L
        check(lib().b2q_ep_moe_prefill_a2a(
            self.comm.ptr if self.comm else None, x.data_ptr() if T else None, self.wr.data_ptr(),
            *[L[n].data_ptr() for n in ("wg", "sg", "bg", "wu", "su", "bu", "wd", "sd", "bd")],
            out.data_ptr() if T else None, None, None, T, T_max, H, self.E, F, self.k, self.gs, self.bits,
            ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream))
        return out


def _stream():
    return torch.cuda.current_stream().cuda_stream


def a2a_dispatch(x: torch.Tensor, router_weight: torch.Tensor, E: int, k: int, nranks: int):
    """Token-owner phase: (send_x [nranks, T, H], send_meta [nranks, T, 2k] int32,
    send_counts [nranks] int32, pos [T, nranks] int32, idx [T, k] int32, w [T, k] f32).
    Block d's first send_counts[d] rows go to rank d."""
    T, H = x.shape
    dev = x.device
    send_x = torch.empty((nranks, T, H), dtype=torch.bfloat16, device=dev)
    send_meta = torch.empty((nranks, T, 2 * k), dtype=torch.int32, device=dev)
    counts = torch.empty((nranks,), dtype=torch.int32, device=dev)
    pos = torch.empty((T, nranks), dtype=torch.int32, device=dev)
    idx = torch.empty((T, k), dtype=torch.int32, device=dev)
    w = torch.empty((T, k), dtype=torch.float32, device=dev)
    size = lib().b2q_ep_a2a_dispatch_workspace_size(max(T, 1), H, E, k, nranks)
    if size == 0:
        raise ValueError("ep a2a dispatch: bad shape")
    ws = torch.zeros(size, dtype=torch.uint8, device=dev)
    ptr = (lambda t: t.data_ptr() if T else None)
    check(lib().b2q_ep_a2a_dispatch(ptr(x), router_weight.data_ptr(), ptr(send_x), ptr(send_meta), counts.data_ptr(),
                                    ptr(pos), ptr(idx), ptr(w), T, H, E, k, nranks, ws.data_ptr(), ws.numel(),
                                    _stream()))
    return send_x, send_meta, counts, pos, idx, w


def a2a_experts(recv_x: torch.Tensor, recv_meta: torch.Tensor, local_layer: dict, E: int, e_lo: int, k: int,
                group_size: int = 64, bits: int = 4) -> torch.Tensor:
    """Expert-rank phase: the fp32 partial rows [R, H] of the received rows."""
    R, H = recv_x.shape
    F = local_layer["wg"].shape[1]
    e_local = local_layer["wg"].shape[0]
    partial = torch.empty((R, H), dtype=torch.float32, device=recv_x.device)
    if R == 0:
        return partial
    ws = torch.zeros(lib().b2q_ep_a2a_experts_workspace_size(R, H, E, F, k), dtype=torch.uint8, device=recv_x.device)
    L = local_layer
    check(lib().b2q_ep_a2a_experts(recv_x.data_ptr(), recv_meta.data_ptr(),
                                   *[L[n].data_ptr() for n in ("wg", "sg", "bg", "wu", "su", "bu", "wd", "sd", "bd")],
                                   partial.data_ptr(), R, H, E, F, k, e_lo, e_local, group_size, bits, ws.data_ptr(),
                                   ws.numel(), _stream()))
    return partial


def a2a_combine(ret: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
    """Token-owner phase: ret [nranks, T, H] fp32 (block d = the rows rank d returned)
    -> out [T, H] bf16."""
    nranks, T, H = ret.shape
    out = torch.empty((T, H), dtype=torch.bfloat16, device=ret.device)
    if T:
        check(lib().b2q_ep_a2a_combine(ret.data_ptr(), pos.data_ptr(), out.data_ptr(), T, H, nranks, _stream()))
    return out
