"""Oracle routing / sort / epilogue semantics (CPU).

Tie rule and softmax of TrackFastMoE.swift:767-911, the stable expert sort of
TrackPrefillSort.swift:17-44, mlx_colsum_small_f32 and the bf16 Sigmoid of
TrackFastKernels2.swift:22-47.
"""
from __future__ import annotations

import numpy as np

from oracle.oracle import bf16_to_f32, f32_to_bf16


def test_route_ties_go_to_lower_index(oracle):
    lg = np.zeros((1, 64), np.float32)
    lg[0, [5, 9, 40, 41]] = 2.0
    lg[0, [3, 63]] = 1.0
    idx, w = oracle.route(lg, 6)
    assert idx.tolist() == [[5, 9, 40, 41, 3, 63]]
    assert abs(w.sum() - 1.0) < 1e-6
    assert np.allclose(w[0, :4], w[0, 0]) and np.allclose(w[0, 4:], w[0, 4])


def test_route_descending_and_softmax(oracle):
    rng = np.random.default_rng(0)
    lg = rng.standard_normal((5, 128)).astype(np.float32)
    idx, w = oracle.route(lg, 8)
    for t in range(5):
        order = np.argsort(-lg[t], kind="stable")[:8]
        assert idx[t].tolist() == order.tolist()
        sel = lg[t, order].astype(np.float64)
        ref = np.exp(sel - sel.max())
        ref /= ref.sum()
        assert np.allclose(w[t], ref, rtol=1e-6, atol=1e-7)


def test_sort_is_the_stable_permutation(oracle):
    rng = np.random.default_rng(3)
    T, k, E = 37, 8, 16
    ids = rng.integers(0, E, size=(T, k)).astype(np.uint32)
    sids, rows, inv, offs = oracle.sort_by_expert(ids, E, k)
    order = np.argsort(ids.ravel(), kind="stable")
    assert np.array_equal(sids, ids.ravel()[order])
    assert np.array_equal(rows, (order // k).astype(np.uint32))
    assert np.array_equal(inv[order], np.arange(T * k))
    assert offs[0] == 0 and offs[-1] == T * k
    assert np.array_equal(np.diff(offs.astype(np.int64)), np.bincount(ids.ravel(), minlength=E))


def test_colsum_small_association(oracle):
    r = np.array([1e8, 1.0, -1e8, 1.0, 3.0, 5.0, 7.0, 9.0, 11.0, 13.0], np.float32)
    # TY = 8 chains: t[y] = r[y] (+ r[y+8]), folded as t[j] + total in order
    t = [np.float32(0)] * 8
    for y in range(8):
        acc = np.float32(0)
        for q in range(y, 10, 8):
            acc = np.float32(r[q] + acc)
        t[y] = acc
    tot = t[0]
    for j in range(1, 8):
        tot = np.float32(t[j] + tot)
    assert oracle.colsum_small(r) == float(tot)


def test_sigmoid_silu_bf16(oracle):
    xs = f32_to_bf16(np.array([-8.0, -1.0, -0.0, 0.0, 0.5, 1.0, 3.0, 20.0], np.float32))
    sg = bf16_to_f32(oracle.sigmoid(xs))
    ref = 1.0 / (1.0 + np.exp(-bf16_to_f32(xs).astype(np.float64)))
    assert np.allclose(sg, ref, atol=4e-3)
    # silu(0) = 0 and swiglu(g, 0) = 0 exactly
    z = f32_to_bf16(np.zeros(1, np.float32))
    assert bf16_to_f32(oracle.swiglu(z, xs[:1]))[0] == 0.0


def test_moe_decode_composes(oracle):
    """The fused oracle equals its own pieces (router -> route -> experts)."""
    rng = np.random.default_rng(11)
    E, H, F, k, gs = 8, 512, 256, 2, 64

    def pw(rows, K):
        w = rng.integers(0, 2**32, size=(*rows, K // 8), dtype=np.uint64).astype(np.uint32)
        s = f32_to_bf16(rng.uniform(0.002, 0.02, (*rows, K // gs)).astype(np.float32))
        b = f32_to_bf16(-8 * bf16_to_f32(s) + rng.normal(0, 1e-3, s.shape).astype(np.float32))
        return w, s, b

    L = {}
    L["wg"], L["sg"], L["bg"] = pw((E, F), H)
    L["wu"], L["su"], L["bu"] = pw((E, F), H)
    L["wd"], L["sd"], L["bd"] = pw((E, H), F)
    x = f32_to_bf16(rng.standard_normal((2, H)).astype(np.float32))
    wr = f32_to_bf16(rng.normal(0, 0.02, (E, H)).astype(np.float32))
    r = oracle.moe_decode(x, wr, L, k, gs)
    lg = oracle.router_logits(x, wr)
    assert np.array_equal(lg, r["logits"])
    idx, w = oracle.route(lg, k)
    assert np.array_equal(idx, r["idx"]) and np.array_equal(w, r["w"])
    out = oracle.moe_experts_decode(x, idx, w, L, k, gs)
    assert np.array_equal(out, r["out"])
