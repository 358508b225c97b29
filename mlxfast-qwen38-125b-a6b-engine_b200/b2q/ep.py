"""Expert parallelism: experts sharded over the ranks of a process group.

The reference's expert-parallel configuration of its MoE layer: every rank
holds the router and a contiguous block of experts, computes the routing in
full, multiplies the selected experts it holds and sums its weighted outputs
into an fp32 partial; one all-reduce of the partial per layer gives the layer
output (NCCL, inside the library, on the caller's stream).

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
    """(e_lo, e_local) of `rank`: contiguous blocks, the first E % world ranks one larger."""
    if not (0 <= rank < world) or E < world:
        raise ValueError(f"cannot shard {E} experts over {world} ranks")
    base, extra = divmod(E, world)
    e_lo = rank * base + min(rank, extra)
    return e_lo, base + (1 if rank < extra else 0)


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
