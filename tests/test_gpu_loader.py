"""A layer bound from a safetensors checkpoint (device copies of the stored
bytes) gives the same MoE output, bit for bit, as the tensors it was written from."""
from __future__ import annotations

import pytest

pytestmark = pytest.mark.gpu


def test_layer_from_checkpoint_matches(tmp_path, cuda, b2q_mod):
    import torch

    from b2q import synth
    from b2q.loader import SafetensorsFile, load_moe_layer, save_safetensors

    E, H, F, k = 16, 1024, 512, 4
    L = synth.moe_layer(E, H, F, 64, seed=110)
    wr = synth.router_weight(E, H, seed=111)
    prefix = "model.layers.0.mlp"
    names = {"g": "gate_proj", "u": "up_proj", "d": "down_proj"}
    t = {f"{prefix}.gate.weight": wr}
    for short, proj in names.items():
        for kind, pre in (("weight", "w"), ("scales", "s"), ("biases", "b")):
            t[f"{prefix}.switch_mlp.{proj}.{kind}"] = L[pre + short]
    path = str(tmp_path / "layer.safetensors")
    save_safetensors(path, t)
    with SafetensorsFile(path) as f:
        router, layer = load_moe_layer([f], prefix)
    x = synth.activations((1, H), seed=112)
    a = b2q_mod.moe_decode(x, wr, L, k)
    b = b2q_mod.moe_decode(x, router, layer, k)
    torch.cuda.synchronize()
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))
    xp = synth.activations((64, H), seed=113)
    assert torch.equal(b2q_mod.moe_prefill(xp, wr, L, k).view(torch.int16),
                       b2q_mod.moe_prefill(xp, router, layer, k).view(torch.int16))
