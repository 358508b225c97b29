"""The allocation-free decode entry point (b2q_moe_decode_noalloc).

It runs the one-token fused decode kernel on a scratch array that lives in
the library, for callers that cannot allocate device memory. The GPU test
calls it twice in a row through the C ABI and compares each result with the
workspace-taking entry point (b2q_moe_decode) on the same inputs. The file
sorts last so the test also runs after every other test in one process.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import rel_l2

TIGHT = 5e-3
SCRATCH_BYTES = 131072  # B2Q_NOALLOC_SCRATCH_BYTES in include/b2q.h


def _bf(t):
    from b2q.synth import to_numpy_bits
    from oracle.oracle import bf16_to_f32

    return bf16_to_f32(to_numpy_bits(t))


def test_noalloc_refuses_oversized_shapes(b2q_mod):
    """Checked on the host before any CUDA call: the scratch has a fixed size."""
    lib = b2q_mod.lib()
    assert lib.b2q_moe_decode_workspace_size(1, 4096, 1024, 16384, 8) > SCRATCH_BYTES
    rc = lib.b2q_moe_decode_noalloc(*([None] * 15), 4096, 1024, 16384, 8, 64, 4, None, None)
    assert rc == -1
    assert b"scratch" in lib.b2q_last_error()


@pytest.mark.gpu
def test_noalloc_matches_workspace_decode(cuda, b2q_mod):
    import torch

    from b2q import synth

    lib = b2q_mod.lib()
    E, H, F, k, gs = 128, 4096, 1536, 8, 64
    assert lib.b2q_moe_decode_workspace_size(1, H, E, F, k) <= SCRATCH_BYTES
    L = synth.moe_layer(E, H, F, gs, seed=70)
    wr = synth.router_weight(E, H, seed=71)
    stream = torch.cuda.current_stream().cuda_stream
    ws = torch.zeros(lib.b2q_moe_decode_workspace_size(1, H, E, F, k), dtype=torch.uint8, device="cuda")
    status = torch.full((1,), 7, dtype=torch.int32, device="cuda")
    weights = [L[n].data_ptr() for n in ("wg", "sg", "bg", "wu", "su", "bu", "wd", "sd", "bd")]

    for call, seed in enumerate((72, 73)):
        x = synth.activations((1, H), seed=seed)
        outs = {}
        for form in ("workspace", "noalloc"):
            out = torch.empty((1, H), dtype=torch.bfloat16, device="cuda")
            idx = torch.empty((1, k), dtype=torch.uint32, device="cuda")
            w = torch.empty((1, k), dtype=torch.float32, device="cuda")
            lg = torch.empty((1, E), dtype=torch.float32, device="cuda")
            ptrs = [x.data_ptr(), wr.data_ptr(), *weights, out.data_ptr(), idx.data_ptr(), w.data_ptr(),
                    lg.data_ptr()]
            if form == "workspace":
                rc = lib.b2q_moe_decode(*ptrs, 1, H, E, F, k, gs, 4, ws.data_ptr(), ws.numel(), stream)
            else:
                rc = lib.b2q_moe_decode_noalloc(*ptrs, H, E, F, k, gs, 4, status.data_ptr(), stream)
            assert rc == 0, lib.b2q_last_error()
            torch.cuda.synchronize()
            outs[form] = (out, idx, w)
        (o_ref, i_ref, w_ref), (o, i, w) = outs["workspace"], outs["noalloc"]
        assert int(status.item()) == 0, f"call {call}: device-side status {int(status.item())}"
        assert torch.equal(i, i_ref), f"call {call}: expert selection differs"
        assert torch.allclose(w, w_ref, rtol=2e-6, atol=1e-7)
        e = rel_l2(_bf(o), _bf(o_ref))
        assert e < TIGHT, f"call {call}: rel L2 {e}"
        assert np.isfinite(_bf(o)).all()
    assert lib.b2q_workspace_status(ws.data_ptr(), ws.numel(), stream) == 0
