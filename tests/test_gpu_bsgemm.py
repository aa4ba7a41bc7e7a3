"""The block-scaled tcgen05 grouped GEMM (the default prefill path for MXFP4
experts: E2M1 weights by TMA, E8M0 scales as UE8M0 scale factors, token and
act rows as hi + lo E4M3 parts) vs the CPU oracle and vs the kind::f16
grouped GEMM (needs a B200).

Tolerance: max|y - y_ref| / max|y_ref| <= 1e-2 on bf16 outputs, as for every
expert path; the hi / lo split keeps layer outputs within ~1e-3 of exact
arithmetic, which the tighter check against the f16 GEMM (exact weights and
2^k-scaled f16 rows) bounds at 5e-3.
"""
import pytest
import torch

import oracle
from oracle import adapter
from whallm_b200 import lib, synth
from whallm_b200.layout import Projection
from whallm_b200.moe import Engine, LayerWeights, RouterWeights, SharedExpert

pytestmark = pytest.mark.gpu

TOL = 1e-2
CROSS_TOL = 5e-3
DEV = "cuda"


def rel(y_bits, ref_bits):
    return oracle.max_rel_error(oracle.bf16_to_f32(y_bits), oracle.bf16_to_f32(ref_bits))


def small_layer(layout, E, H, I, seed, gate=lib.SHARED_NONE, limit=0.0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    w13, s13 = synth.mxfp4_projection(E, 2 * I, H, g, DEV)
    w2, s2 = synth.mxfp4_projection(E, H, I, g, DEV)
    shared = None
    if gate != lib.SHARED_NONE:
        a, b = synth.mxfp4_projection(1, 2 * I, H, g, DEV)
        c, d = synth.mxfp4_projection(1, H, I, g, DEV)
        gw = (torch.randn((H,), generator=g, device=DEV) / H ** 0.5).to(torch.bfloat16)
        shared = SharedExpert(Projection.stacked(a, b), Projection.stacked(c, d), gate,
                              gw if gate == lib.SHARED_SIGMOID_GATE else None)
    wr = (torch.randn((E, H), generator=g, device=DEV) / H ** 0.5).to(torch.bfloat16)
    return LayerWeights(layout, H, I, E, Projection.stacked(w13, s13), Projection.stacked(w2, s2), shared=shared,
                        router=RouterWeights(wr, lib.ROUTER_SOFTMAX), swiglu_limit=limit)


@pytest.fixture(scope="module")
def bs_engine():
    eng = Engine(0, max_tokens=1200, hidden=1024, inter=512, experts=16, topk=8, gemv_max_tokens=-1)
    yield eng
    eng.ctx.close()


@pytest.fixture(scope="module")
def f16_engine():
    eng = Engine(0, max_tokens=1200, hidden=1024, inter=512, experts=16, topk=8, gemv_max_tokens=-1,
                 flags=lib.FLAG_F16_GEMM)
    yield eng
    eng.ctx.close()


def _routes(T, E, K, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return torch.stack([torch.randperm(E, generator=g, device=DEV)[:K] for _ in range(T)]).to(torch.int32)


@pytest.mark.parametrize("layout,limit", [(lib.LAYOUT_QWEN_GATE_UP_MXFP4, 0.0), (lib.LAYOUT_DS_W13_MXFP4, 10.0)])
@pytest.mark.parametrize("T", [1, 65, 300])
def test_bs_gemm_expert_pairs_match_oracle(bs_engine, layout, limit, T):
    """Gate-first (Qwen gate_up) and up-first (w13 = [w3; w1]) weights, the
    SwiGLU clamp, one token up to several 128-row tiles per expert."""
    E, H, I, K = 16, 512, 512, 4
    layer = small_layer(layout, E, H, I, seed=40 + layout, limit=limit)
    x = synth.activations(T, H, torch.Generator(device=DEV).manual_seed(41 + T), DEV)
    idx = _routes(T, E, K, 42 + T)
    before = bs_engine.ctx.counters().bs_gemm_calls
    out = bs_engine.expert_pairs(layer, x, idx)
    bs_engine.sync()
    assert bs_engine.ctx.counters().bs_gemm_calls == before + 1
    ref = adapter.from_layer(layer).pairs(adapter.bits(x), idx.cpu().numpy())
    assert rel(adapter.bits(out), ref) <= TOL


def test_bs_gemm_one_expert_many_tiles(bs_engine):
    """1000 rows of one expert: eight 128-row tiles, the last one partial."""
    H, I = 1024, 512
    layer = small_layer(lib.LAYOUT_QWEN_GATE_UP_MXFP4, 1, H, I, seed=50)
    x = synth.activations(1000, H, torch.Generator(device=DEV).manual_seed(51), DEV)
    idx = torch.zeros((1000, 1), dtype=torch.int32, device=DEV)
    out = bs_engine.expert_pairs(layer, x, idx)
    bs_engine.sync()
    ref = adapter.from_layer(layer).pairs(adapter.bits(x), idx.cpu().numpy())
    assert rel(adapter.bits(out), ref) <= TOL


@pytest.mark.parametrize("layout,gate", [(lib.LAYOUT_QWEN_GATE_UP_MXFP4, lib.SHARED_SIGMOID_GATE),
                                         (lib.LAYOUT_DS_W13_MXFP4, lib.SHARED_ONE)])
def test_bs_gemm_forward_matches_f16_gemm_and_oracle(bs_engine, f16_engine, layout, gate):
    """Routed + shared experts through the whole layer: the block-scaled GEMM
    against the oracle and against the kind::f16 GEMM on the same routes."""
    E, H, I, K, T = 16, 1024, 512, 8, 257
    layer = small_layer(layout, E, H, I, seed=60 + layout, gate=gate)
    x = synth.activations(T, H, torch.Generator(device=DEV).manual_seed(61), DEV)
    before = f16_engine.ctx.counters()
    out_a, (w, idx) = bs_engine.forward(layer, x, K, return_routes=True)
    out_b = f16_engine.forward(layer, x, K, routes=(w, idx))
    bs_engine.sync()
    f16_engine.sync()
    after = f16_engine.ctx.counters()
    assert after.gemm_calls == before.gemm_calls + 1 and after.bs_gemm_calls == before.bs_gemm_calls
    ref = adapter.from_layer(layer).forward(adapter.bits(x), idx.cpu().numpy(), w.cpu().numpy())
    assert rel(adapter.bits(out_a), ref) <= TOL
    assert rel(adapter.bits(out_b), ref) <= TOL
    assert rel(adapter.bits(out_a), adapter.bits(out_b)) <= CROSS_TOL


def test_bs_gemm_repeat_is_deterministic(bs_engine):
    """Two calls on the same input give the same bits (no races between the
    epilogue's act images and the down GEMM, no stale tile images)."""
    E, H, I, K, T = 16, 1024, 512, 8, 300
    layer = small_layer(lib.LAYOUT_QWEN_GATE_UP_MXFP4, E, H, I, seed=70)
    x = synth.activations(T, H, torch.Generator(device=DEV).manual_seed(71), DEV)
    idx = _routes(T, E, K, 72)
    a = bs_engine.expert_pairs(layer, x, idx).clone()
    b = bs_engine.expert_pairs(layer, x, idx).clone()
    bs_engine.sync()
    assert torch.equal(a, b)


def fp8_layer(E, H, I, seed, gate=lib.SHARED_NONE):
    g = torch.Generator(device=DEV).manual_seed(seed)
    w13, s13 = synth.fp8_projection(E, 2 * I, H, g, DEV)
    w2, s2 = synth.fp8_projection(E, H, I, g, DEV)
    shared = None
    if gate != lib.SHARED_NONE:
        a, b = synth.fp8_projection(1, 2 * I, H, g, DEV)
        c, d = synth.fp8_projection(1, H, I, g, DEV)
        shared = SharedExpert(Projection.stacked(a, b), Projection.stacked(c, d), gate)
    wr = (torch.randn((E, H), generator=g, device=DEV) / H ** 0.5).to(torch.bfloat16)
    return LayerWeights(lib.LAYOUT_W13_FP8_B128, H, I, E, Projection.stacked(w13, s13), Projection.stacked(w2, s2),
                        shared=shared, router=RouterWeights(wr, lib.ROUTER_SOFTMAX))


@pytest.mark.parametrize("T", [1, 65, 300])
def test_fp8_block_scaled_gemm_pairs_match_oracle(bs_engine, T):
    """FP8 experts with fp32 128 x 128 block scales: E4M3 weights straight into
    block-scaled MMAs, each 128-K block's partial scaled in registers."""
    E, H, I, K = 16, 512, 512, 4
    layer = fp8_layer(E, H, I, seed=80 + T)
    x = synth.activations(T, H, torch.Generator(device=DEV).manual_seed(81 + T), DEV)
    idx = _routes(T, E, K, 82 + T)
    before = bs_engine.ctx.counters().bs_gemm_calls
    out = bs_engine.expert_pairs(layer, x, idx)
    bs_engine.sync()
    assert bs_engine.ctx.counters().bs_gemm_calls == before + 1
    ref = adapter.from_layer(layer).pairs(adapter.bits(x), idx.cpu().numpy())
    assert rel(adapter.bits(out), ref) <= TOL


def test_fp8_block_scaled_gemm_forward_matches_f16_gemm(bs_engine, f16_engine):
    """Routed + shared FP8 experts through the layer: the block-scaled FP8 GEMM
    against the oracle and against the kind::f16 GEMM on the same routes.  The
    kind::f16 GEMM rounds every dequantised weight to bf16 as the reference
    does; the block-scaled one multiplies the exact E4M3 values and scales each
    128-K block's sum, so the two differ by that rounding (up to 2^-9 of a
    weight; 5-8e-3 of max|y| with these weights spread over every E4M3 code)
    and the cross-check takes the layer tolerance."""
    E, H, I, K, T = 16, 1024, 512, 8, 257
    layer = fp8_layer(E, H, I, seed=90, gate=lib.SHARED_ONE)
    x = synth.activations(T, H, torch.Generator(device=DEV).manual_seed(91), DEV)
    out_a, (w, idx) = bs_engine.forward(layer, x, K, return_routes=True)
    out_b = f16_engine.forward(layer, x, K, routes=(w, idx))
    bs_engine.sync()
    f16_engine.sync()
    ref = adapter.from_layer(layer).forward(adapter.bits(x), idx.cpu().numpy(), w.cpu().numpy())
    assert rel(adapter.bits(out_a), ref) <= TOL
    assert rel(adapter.bits(out_b), ref) <= TOL
    assert rel(adapter.bits(out_a), adapter.bits(out_b)) <= TOL
