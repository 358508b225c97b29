"""Per-layer binding of MLX-format checkpoints (safetensors), layout unchanged.

Mirrors the reference's layer binding (bindMoE, Runner/FastModel/
TrackFastModel.swift:470-540) for the routed experts and the router: the
stacked expert tensors `<prefix>.switch_mlp.{gate,up,down}_proj.{weight,
scales,biases}` ([E, N, K/8] uint32 and [E, N, K/gs] bf16) and the router
`<prefix>.gate.weight` ([E, H] bf16, or a quantized router that is
dequantized once) are read as stored and placed in device memory; nothing is
repacked. The header reader and the copies are the library's b2q_st_* entry
points.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np
import torch

from ._lib import check, lib

_DTYPES = {"U32": (torch.uint32, 4), "BF16": (torch.bfloat16, 2), "F16": (torch.float16, 2),
           "F32": (torch.float32, 4), "I32": (torch.int32, 4), "U8": (torch.uint8, 1)}


class SafetensorsFile:
    def __init__(self, path: str):
        self.path = path
        self.h = ctypes.c_void_p()
        check(lib().b2q_st_open(os.fsencode(path), ctypes.byref(self.h)))

    def close(self):
        if self.h:
            lib().b2q_st_close(self.h)
            self.h = ctypes.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def __del__(self):
        self.close()

    def names(self) -> list[str]:
        out = []
        buf = ctypes.create_string_buffer(4096)
        for i in range(lib().b2q_st_count(self.h)):
            n = lib().b2q_st_name(self.h, i, buf, len(buf))
            if n < 0:
                check(n)
            if n >= len(buf):
                buf = ctypes.create_string_buffer(n + 1)
                lib().b2q_st_name(self.h, i, buf, len(buf))
            out.append(buf.value.decode())
        return out

    def info(self, name: str):
        dt = ctypes.create_string_buffer(16)
        shape = (ctypes.c_int64 * 8)()
        ndim, nbytes = ctypes.c_int(), ctypes.c_uint64()
        check(lib().b2q_st_info(self.h, name.encode(), dt, 16, shape, 8, ctypes.byref(ndim), ctypes.byref(nbytes)))
        return dt.value.decode(), tuple(shape[i] for i in range(ndim.value)), nbytes.value

    def tensor(self, name: str, device="cuda") -> torch.Tensor:
        dtype, shape, nbytes = self.info(name)
        if dtype not in _DTYPES:
            raise ValueError(f"{name}: dtype {dtype} is not used by the path")
        tdt, esize = _DTYPES[dtype]
        n = int(np.prod(shape)) if shape else 1
        if n * esize != nbytes:
            raise ValueError(f"{name}: {nbytes} bytes do not hold shape {shape} of {dtype}")
        dev = torch.device(device)
        out = torch.empty(shape, dtype=tdt, device=dev)
        if n:
            stream = torch.cuda.current_stream(dev).cuda_stream if dev.type == "cuda" else None
            check(lib().b2q_st_read(self.h, name.encode(), out.data_ptr(), nbytes, 1 if dev.type == "cuda" else 0,
                                    stream))
        return out


def load_moe_layer(files, prefix: str, device="cuda", group_size: int = 64, bits: int = 4):
    """(router bf16 [E, H], layer dict wg/sg/bg/wu/su/bu/wd/sd/bd) of one MoE layer.

    `files`: SafetensorsFile objects (a sharded checkpoint); each tensor is read
    from the file that holds it."""
    where = {}
    for f in files:
        for n in f.names():
            where[n] = f

    def get(name):
        if name not in where:
            raise KeyError(f"{name} is not in the checkpoint")
        return where[name].tensor(name, device)

    layer = {}
    for short, proj in (("g", "gate_proj"), ("u", "up_proj"), ("d", "down_proj")):
        base = f"{prefix}.switch_mlp.{proj}"
        layer["w" + short] = get(base + ".weight")
        layer["s" + short] = get(base + ".scales")
        layer["b" + short] = get(base + ".biases")
        if layer["w" + short].dtype != torch.uint32 or layer["s" + short].dtype != torch.bfloat16:
            raise ValueError(f"{base}: expected uint32 packed weights with bf16 scales/biases")
    rname = f"{prefix}.gate.weight"
    router = get(rname)
    if router.dtype == torch.uint32:  # quantized router: dequantize once (bit-exact tile-loader values)
        from .ops import dequantize

        router = dequantize(router, get(f"{prefix}.gate.scales"), get(f"{prefix}.gate.biases"), group_size, bits)
    elif router.dtype != torch.bfloat16:
        router = router.to(torch.bfloat16)
    return router.contiguous(), layer


def save_safetensors(path: str, tensors: dict, metadata: dict | None = None):
    """Write tensors (torch, any device) in the safetensors layout (for tests and fixtures)."""
    import json
    import struct

    rev = {v[0]: k for k, v in _DTYPES.items()}
    header, blobs, off = {}, [], 0
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    for name, t in tensors.items():
        t = t.detach().contiguous().cpu()
        raw = t.view(torch.uint8).numpy().tobytes() if t.numel() else b""
        header[name] = {"dtype": rev[t.dtype], "shape": list(t.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    h = json.dumps(header).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as fh:
        fh.write(struct.pack("<Q", len(h)))
        fh.write(h)
        for b in blobs:
            fh.write(b)
