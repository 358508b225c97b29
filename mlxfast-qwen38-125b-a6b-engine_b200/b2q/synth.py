"""Seeded synthetic inputs with the configured shapes and value distributions.

The benchmark configurations (no public dataset is involved) specify:
packed nibbles q ~ U{0..15} (uniform uint32 words), scales ~ U(0.002, 0.02)
in bf16, biases = -8*scale + N(0, 1e-3) in bf16, activations x ~ N(0, 1) in
bf16, router weights ~ N(0, 0.02) in bf16, seed 0.
"""
from __future__ import annotations

import torch


def _gen(device, seed):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def packed_weights(rows_shape, K, group_size=64, device="cuda", seed=0):
    """(w uint32 [*rows_shape, K/8], scales bf16 [.., K/gs], biases bf16 [.., K/gs])."""
    g = _gen(device, seed)
    shape = tuple(rows_shape)
    w = torch.randint(-(2**31), 2**31, shape + (K // 8,), generator=g, dtype=torch.int32, device=device)
    w = w.view(torch.uint32)
    s = torch.empty(shape + (K // group_size,), dtype=torch.float32, device=device).uniform_(0.002, 0.02, generator=g)
    s = s.to(torch.bfloat16)
    n = torch.empty(s.shape, dtype=torch.float32, device=device).normal_(0.0, 1e-3, generator=g)
    b = (-8.0 * s.float() + n).to(torch.bfloat16)
    return w, s, b


def activations(shape, device="cuda", seed=1):
    g = _gen(device, seed)
    return torch.empty(tuple(shape), dtype=torch.float32, device=device).normal_(0.0, 1.0, generator=g).to(
        torch.bfloat16)


def router_weight(E, H, device="cuda", seed=2):
    g = _gen(device, seed)
    return torch.empty((E, H), dtype=torch.float32, device=device).normal_(0.0, 0.02, generator=g).to(torch.bfloat16)


def moe_layer(E, H, F, group_size=64, device="cuda", seed=10):
    """Expert stacks of one MoE layer: gate/up [E, F, H/8], down [E, H, F/8]."""
    wg, sg, bg = packed_weights((E, F), H, group_size, device, seed)
    wu, su, bu = packed_weights((E, F), H, group_size, device, seed + 1)
    wd, sd, bd = packed_weights((E, H), F, group_size, device, seed + 2)
    return dict(wg=wg, sg=sg, bg=bg, wu=wu, su=su, bu=bu, wd=wd, sd=sd, bd=bd)


def layer_nbytes(layer: dict) -> int:
    return sum(t.numel() * t.element_size() for t in layer.values())


def to_numpy_bits(t: torch.Tensor):
    """Device tensor -> numpy with the raw bits (bf16 -> uint16, uint32 kept)."""
    t = t.detach().contiguous().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view("uint16")
    if t.dtype == torch.uint32:
        return t.view(torch.int32).numpy().view("uint32")
    return t.numpy()


def from_numpy_bits(a, device="cuda"):
    import numpy as np

    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16)).view(torch.bfloat16).to(device)
    if a.dtype == np.uint32:
        return torch.from_numpy(a.view(np.int32)).view(torch.uint32).to(device)
    return torch.from_numpy(a).to(device)
