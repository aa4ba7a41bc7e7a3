"""The pre-MoE RMSNorm in front of the router and the experts (needs a B200).

xn = bf16((x * rsqrt(mean(x^2) + eps)) * w) (rms_norm_tg,
DeepSeekNative/kernels.metal:443-465; GroupRMSNorm, qwen4_exp.py:93-117),
applied once before the gate (engine.mm:1846).  Short calls normalise inside
the router's logits kernel; long calls and other shapes run the RMSNorm
kernel first.  Checks: xn against the oracle within one bf16 step (the two
sums of squares are added in different orders), the router's logits on the
GPU's xn, and the whole block with a norm bit-identical to the same block
without one fed the GPU's xn.
"""
import numpy as np
import pytest
import torch

import oracle
from oracle import adapter
from whallm_b200 import lib, synth
from whallm_b200.moe import LayerWeights, PreNorm, RouterWeights, SharedExpert
from whallm_b200.layout import Projection

pytestmark = pytest.mark.gpu

TOL = 1e-2
DEV = "cuda"
EPS = 1e-6


def _norm(H: int, seed: int) -> PreNorm:
    g = torch.Generator(device=DEV).manual_seed(seed)
    return PreNorm((1.0 + 0.2 * torch.randn((H,), generator=g, device=DEV)).to(torch.bfloat16), EPS)


def _check_xn(xn: torch.Tensor, x: torch.Tensor, norm: PreNorm) -> np.ndarray:
    """xn within one bf16 step of the oracle everywhere, equal almost everywhere."""
    ref = oracle.rms_norm(adapter.bits(x), adapter.bits(norm.weight), norm.eps)
    got = adapter.bits(xn)
    a, b = oracle.bf16_to_f32(got), oracle.bf16_to_f32(ref)
    step = np.maximum(np.abs(b), 1e-30) * 2.0 ** -7
    assert np.all(np.abs(a - b) <= step)
    assert np.mean(got == ref) > 0.99
    return got


def _layer_with_router(H, E, seed, norm=True, shared=lib.SHARED_NONE):
    g = torch.Generator(device=DEV).manual_seed(seed)
    I = 256
    w13, s13 = synth.mxfp4_projection(E, 2 * I, H, g, DEV)
    w2, s2 = synth.mxfp4_projection(E, H, I, g, DEV)
    sh = None
    if shared != lib.SHARED_NONE:
        a, b = synth.mxfp4_projection(1, 2 * I, H, g, DEV)
        c, d = synth.mxfp4_projection(1, H, I, g, DEV)
        gate = (torch.randn((H,), generator=g, device=DEV) / H ** 0.5).to(torch.bfloat16)
        sh = SharedExpert(Projection.stacked(a, b), Projection.stacked(c, d), shared,
                          gate if shared == lib.SHARED_SIGMOID_GATE else None)
    wr = (torch.randn((E, H), generator=g, device=DEV) / H ** 0.5).to(torch.bfloat16)
    return LayerWeights(lib.LAYOUT_QWEN_GATE_UP_MXFP4, H, I, E, Projection.stacked(w13, s13),
                        Projection.stacked(w2, s2), shared=sh, router=RouterWeights(wr, lib.ROUTER_SOFTMAX),
                        norm=_norm(H, seed + 1) if norm else None)


def _without_norm(layer: LayerWeights) -> LayerWeights:
    return LayerWeights(layer.layout, layer.H, layer.I, layer.E, layer.w13, layer.w2, shared=layer.shared,
                        router=layer.router, swiglu_limit=layer.swiglu_limit)


# T = 1 / 37: the fused logits kernel (H % 512 == 0); T = 300: the RMSNorm
# kernel, then the tcgen05 logits GEMM; H = 576: the RMSNorm kernel, then the
# CUDA-core logits kernel
@pytest.mark.parametrize("T,H", [(1, 2048), (37, 2048), (300, 2048), (37, 576)])
def test_router_on_normalised_rows(engine_factory, T, H):
    E, K = 128, 6
    layer = _layer_with_router(H, E, seed=5 + T)
    eng = engine_factory(512, 2048, 512, 512, 10)
    x = synth.activations(T, H, torch.Generator(device=DEV).manual_seed(T), DEV)
    x = x * 3.0  # rows far from unit RMS, so the norm matters
    x = x.to(torch.bfloat16)
    xn = torch.empty_like(x)
    w, idx, logits = eng.route(layer, x, K, with_logits=True, x_norm=xn)
    eng.sync()
    got = _check_xn(xn, x, layer.norm)
    ref_logits = oracle.router_logits(got, adapter.bits(layer.router.weight))
    np.testing.assert_allclose(logits.cpu().numpy(), ref_logits, rtol=2e-5, atol=2e-5)
    oi, ow = oracle.route(lib.ROUTER_SOFTMAX, logits.cpu().numpy(), K)
    np.testing.assert_array_equal(idx.cpu().numpy(), oi)
    np.testing.assert_allclose(w.cpu().numpy(), ow, rtol=1e-5, atol=1e-7)


@pytest.mark.parametrize("T", [1, 24, 300])
@pytest.mark.parametrize("gate", [lib.SHARED_SIGMOID_GATE, lib.SHARED_ONE])
def test_forward_with_norm_is_forward_of_normalised_rows(engine_factory, T, gate):
    """The block with a norm weight equals, bit for bit, the block without one
    given the normalised rows -- and that block matches the oracle."""
    H, E, K = 2048, 128, 6
    layer = _layer_with_router(H, E, seed=90 + T, shared=gate)
    eng = engine_factory(512, 2048, 512, 512, 10)
    x = synth.activations(T, H, torch.Generator(device=DEV).manual_seed(91 + T), DEV)
    xn = torch.empty_like(x)
    out, (w, idx) = eng.forward(layer, x, K, return_routes=True, x_norm=xn)
    eng.sync()
    got = _check_xn(xn, x, layer.norm)
    out2, (w2, idx2) = eng.forward(_without_norm(layer), xn.clone(), K, return_routes=True)
    eng.sync()
    assert torch.equal(idx, idx2) and torch.equal(w, w2)
    assert torch.equal(out.view(torch.int16), out2.view(torch.int16))
    ref = adapter.from_layer(layer).forward(got, idx.cpu().numpy(), w.cpu().numpy())
    assert oracle.max_rel_error(oracle.bf16_to_f32(adapter.bits(out)), oracle.bf16_to_f32(ref)) <= TOL


def test_forward_with_norm_keeps_xn_in_the_workspace(engine_factory):
    """Without x_norm the result is the same (xn stays in the handle's workspace)."""
    H, E, K, T = 2048, 64, 6, 8
    layer = _layer_with_router(H, E, seed=41, shared=lib.SHARED_SIGMOID_GATE)
    eng = engine_factory(512, 2048, 512, 512, 10)
    x = synth.activations(T, H, torch.Generator(device=DEV).manual_seed(42), DEV)
    xn = torch.empty_like(x)
    a = eng.forward(layer, x, K, x_norm=xn)
    b = eng.forward(layer, x, K)
    eng.sync()
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))


def test_given_routes_and_pairs_with_norm(engine_factory):
    H, E, K, T = 2048, 64, 4, 9
    layer = _layer_with_router(H, E, seed=61)
    eng = engine_factory(512, 2048, 512, 512, 10)
    x = synth.activations(T, H, torch.Generator(device=DEV).manual_seed(62), DEV)
    g = torch.Generator(device=DEV).manual_seed(63)
    idx = torch.stack([torch.randperm(E, generator=g, device=DEV)[:K] for _ in range(T)]).to(torch.int32)
    w = torch.full((T, K), 0.25, dtype=torch.float32, device=DEV)
    xn = torch.empty_like(x)
    out = eng.forward(layer, x, K, routes=(w, idx), x_norm=xn)
    pairs = eng.expert_pairs(layer, x, idx)
    eng.sync()
    _check_xn(xn, x, layer.norm)
    plain = _without_norm(layer)
    assert torch.equal(out.view(torch.int16), eng.forward(plain, xn, K, routes=(w, idx)).view(torch.int16))
    assert torch.equal(pairs.view(torch.int16), eng.expert_pairs(plain, xn, idx).view(torch.int16))
    eng.sync()


def test_norm_argument_errors(engine_factory):
    H, E, K, T = 2048, 64, 4, 4
    layer = _layer_with_router(H, E, seed=71)
    eng = engine_factory(512, 2048, 512, 512, 10)
    x = synth.activations(T, H, torch.Generator(device=DEV).manual_seed(72), DEV)
    with pytest.raises(lib.WMError, match="overlap"):
        eng.forward(layer, x, K, x_norm=x)
    with pytest.raises(ValueError, match="pre-MoE norm"):
        eng.forward(_without_norm(layer), x, K, x_norm=torch.empty_like(x))
    bad = LayerWeights(layer.layout, H, layer.I, E, layer.w13, layer.w2, router=layer.router,
                       norm=PreNorm(layer.norm.weight, -1.0))
    with pytest.raises(lib.WMError, match="norm_eps"):
        eng.forward(bad, x, K)
