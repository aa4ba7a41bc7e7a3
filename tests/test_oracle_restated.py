"""The C oracle's routers, expert FFN and combine against a second, independent
restatement in numpy written from the reference's own code (CPU only).

The oracle (oracle/wm_oracle.c) is the checker of every GPU parity test; the
layer arithmetic behind mx.gather_qmm cannot run here, so these tests guard
the checker itself: the same reference semantics, restated a second time in
float64 numpy, must give the same routes and the same bf16 rows.

  softmax router, renormalised top-k   runtime/deepseek_v4_ssd/qwen4_exp.py:1009-1047
  sqrt-softplus / sigmoid + bias gate  runtime/deepseek_v4_ssd/deepseek_v41/moe.py:58-74
  sigmoid + correction bias            runtime/deepseek_v4_ssd/mimo/model.py:139-150
  E2M1 table, E8M0 = 2^(b - 127)       runtime/deepseek_v4_ssd/deepseek_v41/dequant.py:27-68
  SwiGLU (clamped for V4.1)            qwen4_exp.py:815-818, deepseek_v41/moe.py:30-43
  weighted sum of the expert rows      qwen4_exp.py:1049-1051
"""
import numpy as np
import pytest

import oracle

E2M1 = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, 0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0])


def bf16(v):
    """float64 -> the bf16 value nearest its float32 rounding (the oracle's two-step rounding)."""
    return oracle.bf16_to_f32(oracle.f32_to_bf16(np.asarray(v, dtype=np.float32))).astype(np.float64)


def dequant(packed, scales):
    """Packed E2M1 [rows, cols/2] (low nibble = even column) + E8M0 [rows, cols/32] -> float64."""
    lo, hi = packed & 0x0F, packed >> 4
    vals = np.stack([E2M1[lo], E2M1[hi]], axis=-1).reshape(packed.shape[0], -1)
    return vals * np.repeat(np.exp2(scales.astype(np.float64) - 127.0), 32, axis=1)


def route_numpy(kind, logits, K, bias=None, route_scale=1.0):
    """(indices as sets per row, {expert: weight} per row) from the reference's formulas."""
    l = logits.astype(np.float64)
    if kind == oracle.ROUTER_SOFTMAX:
        p = np.exp(l - l.max(axis=1, keepdims=True))
        p /= p.sum(axis=1, keepdims=True)
        idx = np.argsort(-p, axis=1, kind="stable")[:, :K]
        w = np.take_along_axis(p, idx, axis=1)
        w = w / w.sum(axis=1, keepdims=True)  # norm_topk_prob
    else:
        s = np.sqrt(np.logaddexp(0.0, l)) if kind == oracle.ROUTER_SQRTSOFTPLUS else 1.0 / (1.0 + np.exp(-l))
        biased = s + (0.0 if bias is None else bias.astype(np.float64))
        idx = np.argsort(-biased, axis=1, kind="stable")[:, :K]
        w = np.take_along_axis(s, idx, axis=1)  # the bias picks experts but does not scale them
        if K > 1:
            w = w / (w.sum(axis=1, keepdims=True) + 1e-20)
        w = w * route_scale
    return idx, w


@pytest.mark.parametrize("kind,E,K,biased,scale", [
    (oracle.ROUTER_SOFTMAX, 512, 10, False, 1.0),
    (oracle.ROUTER_SOFTMAX, 64, 1, False, 1.0),
    (oracle.ROUTER_SQRTSOFTPLUS, 256, 6, True, 2.5),
    (oracle.ROUTER_SIGMOID, 384, 8, True, 1.0),
    (oracle.ROUTER_SIGMOID, 128, 1, False, 1.0),
])
def test_oracle_routes_match_the_numpy_restatement(kind, E, K, biased, scale):
    rng = np.random.default_rng(E + K + kind)
    logits = rng.standard_normal((64, E)).astype(np.float32)
    bias = (0.1 * rng.standard_normal(E)).astype(np.float32) if biased else None
    oi, ow = oracle.route(kind, logits, K, bias, 1, 1, scale)
    ni, nw = route_numpy(kind, logits, K, bias, scale)
    for t in range(logits.shape[0]):
        assert set(oi[t].tolist()) == set(ni[t].tolist())
        got = dict(zip(oi[t].tolist(), ow[t].tolist()))
        want = dict(zip(ni[t].tolist(), nw[t].tolist()))
        for e in want:
            assert got[e] == pytest.approx(want[e], rel=1e-5, abs=1e-7)
    # the oracle lists a token's selections in descending key order
    keys = logits if kind == oracle.ROUTER_SOFTMAX else None
    if keys is not None:
        sel = np.take_along_axis(keys, oi, axis=1)
        assert np.all(np.diff(sel, axis=1) <= 0)


def test_oracle_group_limited_routes_match_the_numpy_restatement():
    """The group-limited sigmoid router (config 3; not in the reference): a
    group's score is the sum of its two largest biased scores, the best
    topk_groups groups stay eligible, then the top-k of biased scores among
    them, weighted by the unbiased scores."""
    rng = np.random.default_rng(3)
    T, E, K, G, keep, scale = 32, 256, 8, 8, 4, 2.5
    logits = rng.standard_normal((T, E)).astype(np.float32)
    bias = (0.1 * rng.standard_normal(E)).astype(np.float32)
    oi, ow = oracle.route(oracle.ROUTER_SIGMOID_GROUPED, logits, K, bias, G, keep, scale)
    s = 1.0 / (1.0 + np.exp(-logits.astype(np.float64)))
    biased = s + bias
    for t in range(T):
        groups = biased[t].reshape(G, E // G)
        gscore = np.sort(groups, axis=1)[:, -2:].sum(axis=1)
        kept = np.argsort(-gscore, kind="stable")[:keep]
        mask = np.full(E, -np.inf)
        for g in kept:
            mask[g * (E // G):(g + 1) * (E // G)] = 0.0
        sel = np.argsort(-(biased[t] + mask), kind="stable")[:K]
        w = s[t, sel] / (s[t, sel].sum() + 1e-20) * scale
        assert set(oi[t].tolist()) == set(sel.tolist())
        got = dict(zip(oi[t].tolist(), ow[t].tolist()))
        for e, v in zip(sel.tolist(), w.tolist()):
            assert got[e] == pytest.approx(v, rel=1e-5, abs=1e-7)


def ffn_numpy(layout, x, w13, s13, w2, s2, limit):
    """One expert on float rows x [R, H]: bf16 gate/up products, bf16 SwiGLU, bf16 down rows."""
    W13, W2 = dequant(w13, s13), dequant(w2, s2)
    I = W2.shape[1]
    gu = x @ W13.T
    first, second = bf16(gu[:, :I]), bf16(gu[:, I:])
    g, u = (first, second) if layout == oracle.LAYOUT_QWEN_GATE_UP_MXFP4 else (second, first)
    if limit > 0:
        g, u = np.minimum(g, limit), np.clip(u, -limit, limit)
    act = bf16(g / (1.0 + np.exp(-g)) * u)
    return bf16(act @ W2.T)


def _experts(rng, E, H, I):
    w13 = rng.integers(0, 256, size=(E, 2 * I, H // 2), dtype=np.uint8)
    s13 = rng.integers(118, 124, size=(E, 2 * I, H // 32), dtype=np.uint8)
    w2 = rng.integers(0, 256, size=(E, H, I // 2), dtype=np.uint8)
    s2 = rng.integers(118, 124, size=(E, H, I // 32), dtype=np.uint8)
    return w13, s13, w2, s2


def _close_in_bf16(got_bits, want):
    """Equal bf16 bits almost everywhere, never more than one bf16 step apart."""
    got = oracle.bf16_to_f32(got_bits).astype(np.float64)
    step = np.maximum(np.abs(want), 1e-30) * 2.0 ** -7
    assert np.all(np.abs(got - want) <= step)
    assert np.mean(got == want) > 0.99


@pytest.mark.parametrize("layout,limit", [(oracle.LAYOUT_QWEN_GATE_UP_MXFP4, 0.0),
                                          (oracle.LAYOUT_DS_W13_MXFP4, 10.0)])
def test_oracle_expert_rows_match_the_numpy_restatement(layout, limit):
    rng = np.random.default_rng(11 + layout)
    E, H, I, T, K = 6, 256, 128, 12, 3
    w13, s13, w2, s2 = _experts(rng, E, H, I)
    layer = oracle.Layer(layout, H, I, w13, s13, w2, s2, swiglu_limit=limit)
    x_bits = oracle.f32_to_bf16(rng.standard_normal((T, H)).astype(np.float32))
    idx = np.stack([rng.permutation(E)[:K] for _ in range(T)]).astype(np.int32)
    got = layer.pairs(x_bits, idx)
    x = oracle.bf16_to_f32(x_bits).astype(np.float64)
    for e in range(E):
        t, k = np.nonzero(idx == e)
        if t.size == 0:
            continue
        want = ffn_numpy(layout, x[t], w13[e], s13[e], w2[e], s2[e], limit)
        _close_in_bf16(got[t, k], want)


def test_oracle_combine_is_the_fp32_weighted_sum_in_k_order():
    rng = np.random.default_rng(5)
    E, H, I, T, K = 8, 256, 128, 10, 4
    w13, s13, w2, s2 = _experts(rng, E, H, I)
    layer = oracle.Layer(oracle.LAYOUT_QWEN_GATE_UP_MXFP4, H, I, w13, s13, w2, s2)
    x_bits = oracle.f32_to_bf16(rng.standard_normal((T, H)).astype(np.float32))
    idx = np.stack([rng.permutation(E)[:K] for _ in range(T)]).astype(np.int32)
    w = rng.random((T, K)).astype(np.float32)
    rows = oracle.bf16_to_f32(layer.pairs(x_bits, idx))
    acc = np.zeros((T, H), np.float32)
    for k in range(K):  # fp32 products and sums, k order
        acc = (acc + w[:, k:k + 1] * rows[:, k]).astype(np.float32)
    assert np.array_equal(layer.forward(x_bits, idx, w), oracle.f32_to_bf16(acc))


def dequant_fp8_b128(codes, scales):
    """E4M3 [rows, cols] x fp32 scale per 128 x 128 block, one fp32 product, then bf16
    (mimo/weights.py:17-43: the fp32 product rounded to the bf16 weight)."""
    import torch
    v = torch.from_numpy(codes).view(torch.float8_e4m3fn).to(torch.float32).numpy()
    s = np.repeat(np.repeat(scales, 128, axis=0), 128, axis=1)[:codes.shape[0], :codes.shape[1]]
    return bf16((v * s).astype(np.float32))


def test_oracle_fp8_expert_rows_match_the_numpy_restatement():
    rng = np.random.default_rng(21)
    E, H, I, T, K = 3, 256, 256, 6, 2
    def codes(shape):
        c = rng.integers(0, 254, size=shape)
        return np.where(c < 127, c, c + 1).astype(np.uint8)  # no NaN codes (0x7F, 0xFF)
    w13, w2 = codes((E, 2 * I, H)), codes((E, H, I))
    s13 = (rng.random((E, 2 * I // 128, H // 128)) * 2 ** -6 + 2 ** -8).astype(np.float32)
    s2 = (rng.random((E, H // 128, I // 128)) * 2 ** -6 + 2 ** -8).astype(np.float32)
    layer = oracle.Layer(oracle.LAYOUT_W13_FP8_B128, H, I, w13, s13, w2, s2)
    x_bits = oracle.f32_to_bf16(rng.standard_normal((T, H)).astype(np.float32))
    idx = np.stack([rng.permutation(E)[:K] for _ in range(T)]).astype(np.int32)
    got = layer.pairs(x_bits, idx)
    x = oracle.bf16_to_f32(x_bits).astype(np.float64)
    for e in range(E):
        t, k = np.nonzero(idx == e)
        if t.size == 0:
            continue
        W13, W2 = dequant_fp8_b128(w13[e], s13[e]), dequant_fp8_b128(w2[e], s2[e])
        gu = x[t] @ W13.T
        up, gate = bf16(gu[:, :I]), bf16(gu[:, I:])  # w13 = [w3; w1]: up rows first
        act = bf16(gate / (1.0 + np.exp(-gate)) * up)
        _close_in_bf16(got[t, k], bf16(act @ W2.T))
