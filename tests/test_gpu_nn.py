"""The module-level call sites of b2q.nn on the GPU, against the reference.

QuantizedLinear mirrors MLXNN QuantizedLinear.callAsFunction
(Vendor/mlx-swift/Source/MLXNN/Quantized.swift:336-350): decode rows (M <= 8,
the streaming kernels) and prefill rows (the tcgen05 GEMM), with and without
a bias, against the reference's own MLX CPU kernel in fp32
(backend/cpu/quantized.cpp:341). SwitchLinear against the reference's gather
loop (quantized.cpp:701-747). SwitchGLU (sort, gate / up / down gather_qmm,
SwiGLU, unsort; Runner/FastModel/TrackP12Prefill.swift:198-237) per slot
against the same products chained with the Runner's bf16 rounding points.
MoE decode and prefill windows against the oracle layer.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import rel_l2

pytestmark = pytest.mark.gpu

TIGHT = 5e-3


def _np(t):
    from b2q.synth import to_numpy_bits

    return to_numpy_bits(t)


def _bf(a):
    from oracle.oracle import bf16_to_f32

    return bf16_to_f32(a)


def _f2bf(a):
    from oracle.oracle import f32_to_bf16

    return f32_to_bf16(np.asarray(a, np.float32))


@pytest.fixture(scope="module")
def ref():
    from oracle.oracle import MlxRef

    if not MlxRef.available():
        pytest.fail("oracle/_ref/libmlxref.so (the reference's CPU kernels) is missing on this box")
    r = MlxRef()
    if not r.has_f32:
        pytest.fail("the reference library lacks the fp32 entry points; rebuild oracle/ with REFERENCE set")
    return r


@pytest.mark.parametrize("M", [1, 5, 40])
@pytest.mark.parametrize("with_bias", [False, True])
def test_quantized_linear(cuda, b2q_mod, ref, M, with_bias):
    import torch

    from b2q import synth
    from b2q.nn import QuantizedLinear

    N, K = 384, 2048
    w, s, b = synth.packed_weights((N,), K, 64, seed=90 + M)
    bias = (0.1 * torch.randn(N, device="cuda")).to(torch.bfloat16) if with_bias else None
    lin = QuantizedLinear(w, s, b, 64, 4, bias=bias)
    assert lin.rows == N
    x = synth.activations((M, K), seed=91)
    y = lin(x)
    assert tuple(y.shape) == (M, N) and y.dtype == torch.bfloat16
    yr = ref.qmm_f32(_np(x), _np(w), _np(s), _np(b), 64)
    if with_bias:
        # the bias add of the reference module: bf16 product + bf16 bias, one rounding
        yr = _bf(_f2bf(_bf(_f2bf(yr)) + _bf(_np(bias))[None, :]))
    assert rel_l2(_bf(_np(y)), yr) < TIGHT


def test_quantized_linear_from_linear(cuda, b2q_mod, oracle):
    """from_linear quantizes a bf16 matrix with the GPU quantize (bit-exact to the
    reference's quantize) and multiplies with it."""
    import torch

    from b2q.nn import QuantizedLinear

    g = torch.Generator(device="cuda")
    g.manual_seed(92)
    wf = (0.05 * torch.randn((256, 1024), generator=g, device="cuda")).to(torch.bfloat16)
    lin = QuantizedLinear.from_linear(wf, 64, 4)
    wq, s, b = oracle.quantize(_np(wf), 64, 4)
    assert np.array_equal(_np(lin.weight), wq)
    assert np.array_equal(_np(lin.scales), s) and np.array_equal(_np(lin.biases), b)
    x = (torch.randn((1, 1024), generator=g, device="cuda")).to(torch.bfloat16)
    y = lin(x)
    ref = oracle.qmv_metal(_np(x), wq, s, b, 64, 4)
    assert rel_l2(_bf(_np(y)), _bf(ref)) < TIGHT


@pytest.mark.parametrize("T", [3, 24])
def test_switch_linear_against_reference_gather(cuda, b2q_mod, ref, T):
    """Each token row goes through the expert its index names (rows of x
    expanded to [T, 1, K], as SwitchGLU's call site passes them)."""
    import torch

    from b2q import synth
    from b2q.nn import SwitchLinear

    E, N, K = 8, 256, 1024
    w, s, b = synth.packed_weights((E, N), K, 64, seed=93)
    sl = SwitchLinear(w, s, b, 64, 4)
    x = synth.activations((T, 1, K), seed=94)
    rng = np.random.default_rng(95)
    ids = rng.integers(0, E, size=T).astype(np.uint32)
    idx = torch.from_numpy(ids.astype(np.int32)).cuda().view(torch.uint32)
    y = sl(x, idx)
    assert tuple(y.shape) == (T, 1, N)
    yr = ref.gather_qmm(_np(x), _np(w), _np(s), _np(b), np.arange(T, dtype=np.uint32), ids, 64)
    yy = _bf(_np(y))
    for t in range(T):
        assert rel_l2(yy[t], yr[t]) < TIGHT, t


@pytest.mark.parametrize("T", [4, 33])
def test_switch_glu_per_slot_outputs(cuda, b2q_mod, ref, oracle, T):
    """[T, H] tokens and [T, k] indices -> [T, k, H]: slot (t, j) is expert
    idx[t, j]'s down(swiglu(gate(x_t), up(x_t))), each product the reference's
    fp32 kernel rounded to bf16 as the Runner rounds it."""
    import torch

    from b2q import synth
    from b2q.nn import SwitchGLU, SwitchLinear

    E, H, F, k = 8, 512, 1024, 3
    L = synth.moe_layer(E, H, F, 64, seed=96)
    glu = SwitchGLU(SwitchLinear(L["wg"], L["sg"], L["bg"]), SwitchLinear(L["wu"], L["su"], L["bu"]),
                    SwitchLinear(L["wd"], L["sd"], L["bd"]))
    x = synth.activations((T, H), seed=97)
    rng = np.random.default_rng(98)
    ids = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.uint32)
    idx = torch.from_numpy(ids.astype(np.int32)).cuda().view(torch.uint32)
    y = glu(x, idx)
    assert tuple(y.shape) == (T, k, H)
    xs = _np(x)
    Ln = {n: _np(v) for n, v in L.items()}
    yy = _bf(_np(y))
    for t in range(T):
        for j in range(k):
            e = int(ids[t, j])
            g = _f2bf(ref.qmm_f32(xs[t:t + 1], Ln["wg"][e], Ln["sg"][e], Ln["bg"][e], 64))
            u = _f2bf(ref.qmm_f32(xs[t:t + 1], Ln["wu"][e], Ln["su"][e], Ln["bu"][e], 64))
            a = oracle.swiglu(g, u).reshape(1, F)
            d = ref.qmm_f32(a, Ln["wd"][e], Ln["sd"][e], Ln["bd"][e], 64)
            assert rel_l2(yy[t, j], d[0]) < TIGHT, (t, j)


@pytest.mark.parametrize("T", [1, 6, 48])
def test_moe_module_windows(cuda, b2q_mod, oracle, T):
    """b2q.nn.MoE picks the fused one-token call, the decode window operator or
    the sorted prefill operator by window size; all against the oracle layer."""
    from b2q import synth
    from b2q.nn import MoE

    E, H, F, k = 16, 1024, 512, 4
    L = synth.moe_layer(E, H, F, 64, seed=99)
    wr = synth.router_weight(E, H, seed=100)
    moe = MoE(wr, L, k, 64, 4)
    assert moe.num_experts == E
    x = synth.activations((T, H), seed=101)
    out = moe(x)
    out2, idx, w = moe(x, return_routing=True)[:3]
    assert tuple(out.shape) == (T, H)
    Ln = {n: _np(v) for n, v in L.items()}
    ref = (oracle.moe_experts_decode if T <= 8 else oracle.moe_experts_prefill)(_np(x), _np(idx), _np(w), Ln, k)
    assert rel_l2(_bf(_np(out)), _bf(ref)) < TIGHT
    assert rel_l2(_bf(_np(out2)), _bf(ref)) < TIGHT


def test_moe_one_token_into_persistent_output(cuda, b2q_mod, oracle):
    """The prepared one-token call writes a caller's buffer: same result as a
    fresh output, the buffer itself returned (viewed), nothing allocated."""
    import torch

    from b2q import synth
    from b2q.nn import MoE

    E, H, F, k = 16, 1024, 512, 4
    L = synth.moe_layer(E, H, F, 64, seed=102)
    wr = synth.router_weight(E, H, seed=103)
    moe = MoE(wr, L, k, 64, 4)
    buf = torch.empty((1, H), dtype=torch.bfloat16, device="cuda")
    for seed in (104, 105):
        x = synth.activations((1, H), seed=seed)
        y = moe(x, out=buf)
        assert y.data_ptr() == buf.data_ptr()
        assert torch.equal(buf, moe(x))
    with pytest.raises(ValueError):
        moe(synth.activations((2, H), seed=106), out=buf)
