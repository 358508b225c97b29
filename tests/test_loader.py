"""Checkpoint reading for the per-layer binding (CPU): the safetensors header
rules of the reference's reader (Sources/MLXFastCore/Safetensors.swift:75-180)
and bit-exact round trips of the stacked expert tensors."""
from __future__ import annotations

import json
import struct

import pytest


def _layer_cpu(E=4, H=256, F=128, gs=64, seed=0):
    import torch

    g = torch.Generator().manual_seed(seed)

    def packed(rows, K):
        w = torch.randint(-(2**31), 2**31, (E, rows, K // 8), generator=g, dtype=torch.int32).view(torch.uint32)
        s = torch.rand((E, rows, K // gs), generator=g).mul(0.018).add(0.002).to(torch.bfloat16)
        b = (-8.0 * s.float()).to(torch.bfloat16)
        return w, s, b

    L = {}
    for short, (rows, K) in (("g", (F, H)), ("u", (F, H)), ("d", (H, F))):
        L["w" + short], L["s" + short], L["b" + short] = packed(rows, K)
    wr = torch.randn((E, H), generator=g).mul(0.02).to(torch.bfloat16)
    return wr, L


def _write_layer(path, prefix, wr, L):
    from b2q.loader import save_safetensors

    names = {"g": "gate_proj", "u": "up_proj", "d": "down_proj"}
    t = {f"{prefix}.gate.weight": wr}
    for short, proj in names.items():
        for kind, pre in (("weight", "w"), ("scales", "s"), ("biases", "b")):
            t[f"{prefix}.switch_mlp.{proj}.{kind}"] = L[pre + short]
    save_safetensors(path, t, metadata={"format": "mlx"})


def test_round_trip_and_binding(tmp_path, b2q_mod):
    import torch

    from b2q.loader import SafetensorsFile, load_moe_layer

    wr, L = _layer_cpu()
    p = str(tmp_path / "model.safetensors")
    _write_layer(p, "model.layers.3.mlp", wr, L)
    with SafetensorsFile(p) as f:
        names = f.names()
        assert "model.layers.3.mlp.switch_mlp.gate_proj.weight" in names and len(names) == 10
        dt, shape, nbytes = f.info("model.layers.3.mlp.switch_mlp.down_proj.scales")
        assert dt == "BF16" and shape == tuple(L["sd"].shape) and nbytes == L["sd"].numel() * 2
        router, layer = load_moe_layer([f], "model.layers.3.mlp", device="cpu")
    assert torch.equal(router.view(torch.int16), wr.view(torch.int16))
    for k in L:
        a, b = layer[k], L[k]
        assert a.dtype == b.dtype and a.shape == b.shape
        assert torch.equal(a.view(torch.int16 if a.dtype == torch.bfloat16 else torch.int32),
                           b.view(torch.int16 if b.dtype == torch.bfloat16 else torch.int32))


def _raw(path, header_bytes, data=b"", length=None):
    with open(path, "wb") as fh:
        fh.write(struct.pack("<Q", len(header_bytes) if length is None else length))
        fh.write(header_bytes)
        fh.write(data)


@pytest.mark.parametrize("case", ["small", "empty", "huge", "truncated", "not_object", "bad_offsets",
                                  "past_end", "bad_json", "missing_field"])
def test_header_rules(tmp_path, b2q_mod, case):
    from b2q._lib import B2QError
    from b2q.loader import SafetensorsFile

    p = str(tmp_path / "x.safetensors")
    good = {"t": {"dtype": "U8", "shape": [4], "data_offsets": [0, 4]}}
    if case == "small":
        open(p, "wb").write(b"\x01\x02")
    elif case == "empty":
        _raw(p, b"", length=0)
    elif case == "huge":
        _raw(p, b"{}", length=100_000_001)
    elif case == "truncated":
        _raw(p, json.dumps(good).encode(), length=10_000)
    elif case == "not_object":
        _raw(p, b"[1, 2]", b"abcd")
    elif case == "bad_offsets":
        _raw(p, json.dumps({"t": {"dtype": "U8", "shape": [4], "data_offsets": [4, 0]}}).encode(), b"abcd")
    elif case == "past_end":
        _raw(p, json.dumps({"t": {"dtype": "U8", "shape": [8], "data_offsets": [0, 8]}}).encode(), b"abcd")
    elif case == "bad_json":
        _raw(p, b'{"t": {"dtype": "U8", "shape": [4], "data_offsets": [0, 4]', b"abcd")
    elif case == "missing_field":
        _raw(p, json.dumps({"t": {"dtype": "U8", "shape": [4]}}).encode(), b"abcd")
    with pytest.raises(B2QError) as ei:
        SafetensorsFile(p)
    assert ei.value.code == -1


def test_metadata_and_escapes(tmp_path, b2q_mod):
    from b2q.loader import SafetensorsFile

    p = str(tmp_path / "m.safetensors")
    hdr = {"__metadata__": {"k": "v \" \\u00e9"}, "a\\u00e9/b": {"dtype": "U8", "shape": [2, 2], "data_offsets": [0, 4]}}
    _raw(p, json.dumps(hdr).encode(), b"wxyz")
    with SafetensorsFile(p) as f:
        (name,) = f.names()
        assert name == "a\\u00e9/b"
        t = f.tensor(name, device="cpu")
        assert bytes(t.numpy().tobytes()) == b"wxyz"
