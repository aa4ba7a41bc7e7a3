"""CUDA path vs the CPU oracle, through the C ABI (needs a B200).

Tolerance for layer and expert outputs (bf16): max|y - y_ref| / max|y_ref| <= 1e-2
with identical top-k expert index sets; dequantised weights must be bit-exact.
"""
import numpy as np
import pytest
import torch

import oracle
from oracle import adapter
from whallm_b200 import lib, synth
from whallm_b200.moe import LayerWeights, RouterWeights, SharedExpert
from whallm_b200.layout import Projection

pytestmark = pytest.mark.gpu

TOL = 1e-2
DEV = "cuda"


def rel(y_bits, ref_bits):
    return oracle.max_rel_error(oracle.bf16_to_f32(y_bits), oracle.bf16_to_f32(ref_bits))


def same_bits(a: np.ndarray, b: np.ndarray) -> bool:
    """bf16 bit equality, any NaN equal to any NaN."""
    fa, fb = oracle.bf16_to_f32(a), oracle.bf16_to_f32(b)
    nan = np.isnan(fa) & np.isnan(fb)
    return bool(np.all(nan | (a == b)))


# ---------------------------------------------------------------- dequant (bit-exact)

@pytest.mark.parametrize("convention", [oracle.CONV_MLX, oracle.CONV_METAL])
def test_dequant_mxfp4_bit_exact(engine_factory, convention):
    eng = engine_factory(64, 2048, 512, 16, 8)
    g = torch.Generator(device=DEV).manual_seed(11)
    rows, cols = 256, 1024
    w = torch.randint(0, 256, (rows, cols // 2), generator=g, device=DEV, dtype=torch.uint8)
    s = torch.randint(0, 256, (rows, cols // 32), generator=g, device=DEV, dtype=torch.int32).to(torch.uint8)
    out = eng.dequant(lib.FORMAT_MXFP4, w, s, rows, cols, convention)
    eng.sync()
    ref = oracle.dequant_mxfp4(w.cpu().numpy(), s.cpu().numpy(), convention)
    assert same_bits(adapter.bits(out), ref)


def test_dequant_fp8_b128_bit_exact(engine_factory):
    eng = engine_factory(64, 2048, 512, 16, 8)
    g = torch.Generator(device=DEV).manual_seed(12)
    w, s = synth.fp8_projection(1, 384, 512, g, DEV)
    s = s * (1.0 + torch.rand(s.shape, generator=g, device=DEV))  # scales that are not powers of two
    out = eng.dequant(lib.FORMAT_FP8_B128, w[0], s[0].contiguous(), 384, 512)
    eng.sync()
    ref = oracle.dequant_fp8_b128(w[0].cpu().numpy(), s[0].cpu().numpy())
    assert np.array_equal(adapter.bits(out), ref)


def test_dequant_fp8_b32_bit_exact(engine_factory):
    eng = engine_factory(64, 2048, 512, 16, 8)
    g = torch.Generator(device=DEV).manual_seed(13)
    w, _ = synth.fp8_projection(1, 96, 256, g, DEV)
    s = torch.randint(110, 140, (3, 8), generator=g, device=DEV, dtype=torch.int32).to(torch.uint8)
    out = eng.dequant(lib.FORMAT_FP8_B32, w[0], s, 96, 256)
    eng.sync()
    ref = oracle.dequant_fp8_b32(w[0].cpu().numpy(), s.cpu().numpy())
    assert np.array_equal(adapter.bits(out), ref)


def test_dequant_reports_reserved_fp8_codes(engine_factory):
    eng = engine_factory(64, 2048, 512, 16, 8)
    w = torch.full((128, 128), 0x38, dtype=torch.uint8, device=DEV)
    w[5, 7] = 0x7F
    s = torch.ones((1, 1), dtype=torch.float32, device=DEV)
    eng.dequant(lib.FORMAT_FP8_B128, w, s, 128, 128)
    with pytest.raises(lib.WMError, match="NaN"):
        eng.sync()
    eng.sync()  # the handle stays usable


# ---------------------------------------------------------------- routers

ROUTERS = [
    (lib.ROUTER_SOFTMAX, 512, 10, None, 1, 1, 1.0),
    (lib.ROUTER_SQRTSOFTPLUS, 384, 6, "bias", 1, 1, 1.5),
    (lib.ROUTER_SIGMOID, 256, 8, "bias", 1, 1, 1.0),
    (lib.ROUTER_SIGMOID_GROUPED, 256, 8, "bias", 8, 4, 2.5),
    (lib.ROUTER_SIGMOID, 256, 40, "bias", 1, 1, 1.0),  # K > 32: two selections per lane
]


@pytest.mark.parametrize("kind,E,K,bias,groups,topg,scale", ROUTERS)
def test_router_matches_oracle(engine_factory, kind, E, K, bias, groups, topg, scale):
    H, T = 2048, 37
    eng = engine_factory(64, H, 512, E, K)
    g = torch.Generator(device=DEV).manual_seed(21 + kind)
    layer = synth.qwen_layer(E=8, H=H, I=64, device=DEV, seed=3, shared=False, router=False)
    wr = (torch.randn((E, H), generator=g, device=DEV) / H ** 0.5).to(torch.bfloat16)
    b = None if bias is None else (0.1 * torch.randn((E,), generator=g, device=DEV)).float()
    layer = LayerWeights(layer.layout, H, 64, E, layer.w13, layer.w2,
                         router=RouterWeights(wr, kind, b, groups, topg, scale))
    x = synth.activations(T, H, g, DEV)
    w, idx, logits = eng.route(layer, x, K, with_logits=True)
    eng.sync()
    ref_logits = oracle.router_logits(adapter.bits(x), adapter.bits(wr))
    np.testing.assert_allclose(logits.cpu().numpy(), ref_logits, rtol=2e-5, atol=2e-5)
    bn = None if b is None else b.cpu().numpy()
    # selection on the GPU's own logits: identical indices and weights
    oi, ow = oracle.route(kind, logits.cpu().numpy(), K, bn, groups, topg, scale)
    np.testing.assert_array_equal(idx.cpu().numpy(), oi)
    np.testing.assert_allclose(w.cpu().numpy(), ow, rtol=1e-5, atol=1e-7)
    # end to end: identical index sets per token
    ri, _ = oracle.route(kind, ref_logits, K, bn, groups, topg, scale)
    assert [set(r) for r in idx.cpu().numpy().tolist()] == [set(r) for r in ri.tolist()]


@pytest.mark.parametrize("kind,E,K,groups,topg", [(lib.ROUTER_SOFTMAX, 512, 10, 1, 1),
                                                   (lib.ROUTER_SIGMOID_GROUPED, 256, 8, 8, 4),
                                                   (lib.ROUTER_SIGMOID, 384, 8, 1, 1)])
def test_router_tensor_cores_long_call(engine_factory, kind, E, K, groups, topg):
    """T >= 256 takes the tcgen05 logits GEMM; T = 300 leaves a partial 128-row tile."""
    H, T = 2048, 300
    eng = engine_factory(512, H, 512, E, K)
    g = torch.Generator(device=DEV).manual_seed(31 + kind)
    layer = synth.qwen_layer(E=8, H=H, I=64, device=DEV, seed=3, shared=False, router=False)
    wr = (torch.randn((E, H), generator=g, device=DEV) / H ** 0.5).to(torch.bfloat16)
    layer = LayerWeights(layer.layout, H, 64, E, layer.w13, layer.w2,
                         router=RouterWeights(wr, kind, None, groups, topg, 1.0))
    x = synth.activations(T, H, g, DEV)
    w, idx, logits = eng.route(layer, x, K, with_logits=True)
    eng.sync()
    ref_logits = oracle.router_logits(adapter.bits(x), adapter.bits(wr))
    np.testing.assert_allclose(logits.cpu().numpy(), ref_logits, rtol=2e-5, atol=2e-5)
    oi, ow = oracle.route(kind, logits.cpu().numpy(), K, None, groups, topg, 1.0)
    np.testing.assert_array_equal(idx.cpu().numpy(), oi)
    np.testing.assert_allclose(w.cpu().numpy(), ow, rtol=1e-5, atol=1e-7)
    # end to end: identical index sets, except where the reference's K-th and
    # (K+1)-th logits are closer than the two sums' rounding can separate
    ri, _ = oracle.route(kind, ref_logits, K, None, groups, topg, 1.0)
    srt = -np.sort(-ref_logits, axis=1)
    for t in range(T):
        if kind == lib.ROUTER_SOFTMAX and srt[t, K - 1] - srt[t, K] < 1e-4:
            continue
        if kind != lib.ROUTER_SOFTMAX and np.min(np.abs(np.diff(srt[t]))) < 1e-4:
            continue
        assert set(idx[t].tolist()) == set(ri[t].tolist()), t


# ---------------------------------------------------------------- experts and the whole layer

def _small_layer(layout, E, H, I, seed, shared_gate=lib.SHARED_NONE, limit=0.0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    proj = synth.projection_for(layout)
    w13, s13 = proj(E, 2 * I, H, g, DEV)
    w2, s2 = proj(E, H, I, g, DEV)
    sh = [proj(1, 2 * I, H, g, DEV), proj(1, H, I, g, DEV)]
    shared = None
    if shared_gate != lib.SHARED_NONE:
        gate_w = (torch.randn((H,), generator=g, device=DEV) / H ** 0.5).to(torch.bfloat16)
        shared = SharedExpert(Projection.stacked(*sh[0]), Projection.stacked(*sh[1]), shared_gate,
                              gate_w if shared_gate == lib.SHARED_SIGMOID_GATE else None)
    wr = (torch.randn((E, H), generator=g, device=DEV) / H ** 0.5).to(torch.bfloat16)
    return LayerWeights(layout, H, I, E, Projection.stacked(w13, s13), Projection.stacked(w2, s2), shared=shared,
                        router=RouterWeights(wr, lib.ROUTER_SOFTMAX), swiglu_limit=limit)


def test_config0_single_expert_pairs(engine_factory):
    wl = synth.config(0, device=DEV)
    eng = engine_factory(64, 2048, 512, 16, 8)
    idx = torch.zeros((4, 1), dtype=torch.int32, device=DEV)
    out = eng.expert_pairs(wl.layer, wl.x, idx)
    eng.sync()
    ref = adapter.from_layer(wl.layer).pairs(adapter.bits(wl.x), idx.cpu().numpy())
    assert rel(adapter.bits(out), ref) <= TOL


@pytest.mark.parametrize("layout,limit", [(lib.LAYOUT_QWEN_GATE_UP_MXFP4, 0.0), (lib.LAYOUT_DS_W13_MXFP4, 10.0),
                                          (lib.LAYOUT_W13_FP8_B128, 0.0), (lib.LAYOUT_W13_FP8_B32, 0.0)])
@pytest.mark.parametrize("T", [1, 5, 33])
def test_expert_pairs_match_oracle(engine_factory, layout, limit, T):
    E, H, I, K = 16, 512, 256, 4
    layer = _small_layer(layout, E, H, I, seed=31 + layout, limit=limit)
    eng = engine_factory(64, 2048, 512, 16, 8)
    g = torch.Generator(device=DEV).manual_seed(40 + T)
    x = synth.activations(T, H, g, DEV)
    idx = torch.stack([torch.randperm(E, generator=g, device=DEV)[:K] for _ in range(T)]).to(torch.int32)
    out = eng.expert_pairs(layer, x, idx)
    eng.sync()
    ref = adapter.from_layer(layer).pairs(adapter.bits(x), idx.cpu().numpy())
    assert rel(adapter.bits(out), ref) <= TOL


@pytest.mark.parametrize("layout,gate", [(lib.LAYOUT_QWEN_GATE_UP_MXFP4, lib.SHARED_SIGMOID_GATE),
                                         (lib.LAYOUT_DS_W13_MXFP4, lib.SHARED_ONE),
                                         (lib.LAYOUT_W13_FP8_B128, lib.SHARED_ONE),
                                         (lib.LAYOUT_W13_FP8_B32, lib.SHARED_ONE)])
def test_forward_matches_oracle_small(engine_factory, layout, gate):
    E, H, I, K, T = 16, 512, 256, 4, 24
    layer = _small_layer(layout, E, H, I, seed=51 + layout, shared_gate=gate)
    eng = engine_factory(64, 2048, 512, 16, 8)
    x = synth.activations(T, H, torch.Generator(device=DEV).manual_seed(61), DEV)
    out, (w, idx) = eng.forward(layer, x, K, return_routes=True)
    eng.sync()
    ref = adapter.from_layer(layer).forward(adapter.bits(x), idx.cpu().numpy(), w.cpu().numpy())
    assert rel(adapter.bits(out), ref) <= TOL


def test_repeated_experts_and_given_routes(engine_factory):
    E, H, I, K, T = 8, 512, 256, 4, 9
    layer = _small_layer(lib.LAYOUT_QWEN_GATE_UP_MXFP4, E, H, I, seed=71)
    eng = engine_factory(64, 2048, 512, 16, 8)
    x = synth.activations(T, H, torch.Generator(device=DEV).manual_seed(72), DEV)
    idx = torch.full((T, K), 5, dtype=torch.int32, device=DEV)
    idx[:, 1] = 2
    w = torch.full((T, K), 0.25, dtype=torch.float32, device=DEV)
    out = eng.forward(layer, x, K, routes=(w, idx))
    eng.sync()
    ref = adapter.from_layer(layer).forward(adapter.bits(x), idx.cpu().numpy(), w.cpu().numpy())
    assert rel(adapter.bits(out), ref) <= TOL


def test_empty_call_and_bad_expert(engine_factory):
    E, H, I, K = 8, 512, 256, 2
    layer = _small_layer(lib.LAYOUT_QWEN_GATE_UP_MXFP4, E, H, I, seed=81)
    eng = engine_factory(64, 2048, 512, 16, 8)
    x0 = torch.empty((0, H), dtype=torch.bfloat16, device=DEV)
    assert eng.forward(layer, x0, K).shape == (0, H)
    x = synth.activations(3, H, torch.Generator(device=DEV).manual_seed(82), DEV)
    idx = torch.tensor([[0, 1], [2, 99], [3, 4]], dtype=torch.int32, device=DEV)
    w = torch.full((3, K), 0.5, device=DEV)
    eng.forward(layer, x, K, routes=(w, idx))
    with pytest.raises(lib.WMError, match="outside the model"):
        eng.sync()
    with pytest.raises(lib.WMError):
        eng.forward(layer, synth.activations(65, H, torch.Generator(device=DEV).manual_seed(1), DEV), K)


# 1 / 8 / 64: BASELINE config 1; 2, 4, 16: the reference's small-row
# verification batches (READY_VERIFICATION_ROWS = 16, qwen4_exp.py:786-788)
@pytest.mark.parametrize("batch", [1, 2, 4, 8, 16, 64])
def test_config1_decode_layer_matches_oracle(engine_factory, batch):
    wl = synth.config(1, device=DEV, batch=batch)
    eng = engine_factory(64, 2048, 512, 512, 10)
    out, (w, idx) = eng.forward(wl.layer, wl.x, wl.K, return_routes=True)
    eng.sync()
    xb = adapter.bits(wl.x)
    ref_logits = oracle.router_logits(xb, adapter.bits(wl.layer.router.weight))
    ri, rw = oracle.route(oracle.ROUTER_SOFTMAX, ref_logits, wl.K)
    assert [set(r) for r in idx.cpu().numpy().tolist()] == [set(r) for r in ri.tolist()]
    ref = adapter.from_layer(wl.layer).forward(xb, idx.cpu().numpy(), w.cpu().numpy())
    assert rel(adapter.bits(out), ref) <= TOL


# FP8 experts on the register-direct decode kernel (bf16 MMAs; H, I multiples of 512)
@pytest.mark.parametrize("layout", [lib.LAYOUT_W13_FP8_B128, lib.LAYOUT_W13_FP8_B32])
@pytest.mark.parametrize("T", [1, 8, 40])
def test_fp8_decode_kernel_matches_oracle(engine_factory, layout, T):
    E, H, I, K = 16, 1024, 512, 4
    layer = _small_layer(layout, E, H, I, seed=91 + layout, shared_gate=lib.SHARED_ONE)
    eng = engine_factory(64, 2048, 512, 16, 8)
    x = synth.activations(T, H, torch.Generator(device=DEV).manual_seed(92 + T), DEV)
    before = eng.ctx.counters().decode_calls
    out, (w, idx) = eng.forward(layer, x, K, return_routes=True)
    eng.sync()
    assert eng.ctx.counters().decode_calls == before + 1  # the decode kernel ran, not the GEMV
    ref = adapter.from_layer(layer).forward(adapter.bits(x), idx.cpu().numpy(), w.cpu().numpy())
    assert rel(adapter.bits(out), ref) <= TOL
