"""MoE oracle: routing known answers and the block against a composition of
the oracle's own W8A8 product and gelu_new (CPU)."""
import math

import numpy as np
import pytest

import oracle
import synth


def test_route_ties_pick_lower_expert():
    idx, w = oracle.moe_route(np.array([[1, 3, 3, 2], [0, 0, 0, 0]], np.float32), 2, 4, 2)
    assert idx.tolist() == [[1, 2], [0, 1]]
    assert w.tolist() == [[0.5, 0.5], [0.5, 0.5]]


def test_route_softmax_known_answer():
    idx, w = oracle.moe_route(np.array([[0.0, 2.0, math.log(3.0) + 0.0, -5.0]], np.float32), 1, 4, 3)
    assert idx.tolist() == [[1, 2, 0]]
    e = [1.0, float(np.float32(math.exp(np.float32(math.log(3.0)) - 2.0))),
         float(np.float32(math.exp(-2.0)))]
    s = np.float32(np.float32(e[0]) + np.float32(e[1])) + np.float32(e[2])
    assert w[0].tolist() == [float(np.float32(v) / s) for v in e]
    assert abs(float(w.sum()) - 1.0) < 1e-6


def test_route_nan_never_selected_and_all_nan_uniform():
    lg = np.array([[np.nan, -1.0, np.nan, 4.0], [np.nan, np.nan, np.nan, np.nan]], np.float32)
    idx, w = oracle.moe_route(lg, 2, 4, 2)
    assert idx[0].tolist() == [3, 1]
    assert idx[1].tolist() == [0, 1]
    assert w[1].tolist() == [0.5, 0.5]


def test_route_rejects_k_above_experts():
    with pytest.raises(ValueError):
        oracle.moe_route(np.zeros((1, 2), np.float32), 1, 2, 3)


def _quantized(T, D, F, E, seed):
    x, lg, W1, W2, SW1, SW2 = synth.moe_case(T, D, F, E, seed)
    q = [oracle.quantize_int8(W.ravel(), W.shape[-1]) for W in (W1, W2, SW1, SW2)]
    w1, w2 = q[0].data.reshape(E, F, D), q[1].data.reshape(E, D, F)
    sw1, sw2 = q[2].data.reshape(F, D), q[3].data.reshape(D, F)
    return x, lg, (w1, q[0].scales, w2, q[1].scales, sw1, q[2].scales, sw2, q[3].scales)


def _mlp(x, w1, s1, w2, s2):
    R, D = x.shape
    F = w1.shape[0]
    h = oracle.gelu(oracle.qgemm_w8a8(R, D, F, x, w1, s1, None))
    return oracle.qgemm_w8a8(R, F, D, h, w2, s2, None).reshape(R, D)


def test_moe_forward_matches_composition():
    T, D, F, E, k = 12, 64, 96, 6, 2
    x, lg, w = _quantized(T, D, F, E, 11)
    y = oracle.moe_forward(x, lg, *w, k)
    idx, tw = oracle.moe_route(lg, T, E, k)
    w1, s1, w2, s2, sw1, ss1, sw2, ss2 = w
    ref = _mlp(x, sw1, ss1, sw2, ss2)
    for i in range(k):
        out = np.stack([_mlp(x[t:t + 1], w1[e], s1[e * F:(e + 1) * F], w2[e], s2[e * D:(e + 1) * D])[0]
                        for t, e in enumerate(idx[:, i])])
        ref = ref + tw[:, i:i + 1] * out
    assert np.array_equal(y.view(np.uint32), ref.astype(np.float32).view(np.uint32))
