"""The decode kernels vs the CPU oracle (needs a B200): the default
register-direct kernel (weights dequantised in registers into warp MMAs) and
the tcgen05 kernel (weights as the M operand in TMEM), both with f16 operands
under exact power-of-two scaling.

Tolerance as elsewhere: max|y - y_ref| / max|y_ref| <= 1e-2 on bf16 outputs.
"""
import numpy as np
import pytest
import torch

import oracle
from oracle import adapter
from whallm_b200 import lib, synth
from whallm_b200.layout import Projection
from whallm_b200.moe import Engine, LayerWeights, RouterWeights, SharedExpert

pytestmark = pytest.mark.gpu

TOL = 1e-2
DEV = "cuda"
E, H, I = 16, 1024, 512


def rel(y_bits, ref_bits):
    return oracle.max_rel_error(oracle.bf16_to_f32(y_bits), oracle.bf16_to_f32(ref_bits))


def layer(layout=lib.LAYOUT_QWEN_GATE_UP_MXFP4, seed=3, gate=lib.SHARED_NONE, limit=0.0, exp_lo=-8, exp_hi=-2):
    g = torch.Generator(device=DEV).manual_seed(seed)
    w13, s13 = synth.mxfp4_projection(E, 2 * I, H, g, DEV, exp_lo, exp_hi)
    w2, s2 = synth.mxfp4_projection(E, H, I, g, DEV, exp_lo, exp_hi)
    shared = None
    if gate != lib.SHARED_NONE:
        a, b = synth.mxfp4_projection(1, 2 * I, H, g, DEV, exp_lo, exp_hi)
        c, d = synth.mxfp4_projection(1, H, I, g, DEV, exp_lo, exp_hi)
        gw = (torch.randn((H,), generator=g, device=DEV) / H ** 0.5).to(torch.bfloat16)
        shared = SharedExpert(Projection.stacked(a, b), Projection.stacked(c, d), gate,
                              gw if gate == lib.SHARED_SIGMOID_GATE else None)
    wr = (torch.randn((E, H), generator=g, device=DEV) / H ** 0.5).to(torch.bfloat16)
    return LayerWeights(layout, H, I, E, Projection.stacked(w13, s13), Projection.stacked(w2, s2), shared=shared,
                        router=RouterWeights(wr, lib.ROUTER_SOFTMAX), swiglu_limit=limit)


@pytest.fixture(scope="module", params=[0, lib.FLAG_MMA_DECODE], ids=["block_scaled", "mma"])
def eng(request):
    e = Engine(0, max_tokens=64, hidden=H, inter=I, experts=E, topk=8, flags=request.param)
    yield e
    e.ctx.close()


def routes(T, K, seed, experts=E):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return torch.stack([torch.randperm(experts, generator=g, device=DEV)[:K] for _ in range(T)]).to(torch.int32)


@pytest.mark.parametrize("layout,limit", [(lib.LAYOUT_QWEN_GATE_UP_MXFP4, 0.0), (lib.LAYOUT_DS_W13_MXFP4, 10.0)])
@pytest.mark.parametrize("T", [1, 5, 33])
def test_decode_pairs_match_oracle(eng, layout, limit, T):
    lw = layer(layout, seed=5 + T, limit=limit)
    x = synth.activations(T, H, torch.Generator(device=DEV).manual_seed(6 + T), DEV)
    idx = routes(T, 4, 7 + T)
    before = eng.ctx.counters().decode_calls
    out = eng.expert_pairs(lw, x, idx)
    eng.sync()
    assert eng.ctx.counters().decode_calls == before + 1
    ref = adapter.from_layer(lw).pairs(adapter.bits(x), idx.cpu().numpy())
    assert rel(adapter.bits(out), ref) <= TOL


def test_decode_many_rows_per_expert(eng):
    """More than 16 rows of one expert: several token chunks per weight tile."""
    lw = layer(seed=11)
    T = 60
    x = synth.activations(T, H, torch.Generator(device=DEV).manual_seed(12), DEV)
    idx = routes(T, 2, 13, experts=3)  # 120 pairs over 3 experts: about 40 rows each
    out = eng.expert_pairs(lw, x, idx)
    eng.sync()
    ref = adapter.from_layer(lw).pairs(adapter.bits(x), idx.cpu().numpy())
    assert rel(adapter.bits(out), ref) <= TOL


@pytest.mark.parametrize("scale", [1e4, 1e-5])
def test_decode_activation_magnitudes_outside_f16(eng, scale):
    """Rows far above f16's largest or below its smallest normal stay exact
    through the per-row power-of-two prescale."""
    lw = layer(seed=21)
    T = 9
    x = (synth.activations(T, H, torch.Generator(device=DEV).manual_seed(22), DEV).float() * scale).to(torch.bfloat16)
    x[3] *= 64  # rows of different magnitudes in one call
    idx = routes(T, 4, 23)
    out = eng.expert_pairs(lw, x, idx)
    eng.sync()
    ref = adapter.from_layer(lw).pairs(adapter.bits(x), idx.cpu().numpy())
    assert np.isfinite(oracle.bf16_to_f32(adapter.bits(out))).all()
    assert rel(adapter.bits(out), ref) <= TOL


def test_decode_wide_scale_ranges(eng):
    """E8M0 bytes spread over 20 binades within a row (relative f16 scaling)."""
    lw = layer(seed=31, exp_lo=-22, exp_hi=-2)
    T = 7
    x = synth.activations(T, H, torch.Generator(device=DEV).manual_seed(32), DEV)
    idx = routes(T, 4, 33)
    out = eng.expert_pairs(lw, x, idx)
    eng.sync()
    ref = adapter.from_layer(lw).pairs(adapter.bits(x), idx.cpu().numpy())
    assert rel(adapter.bits(out), ref) <= TOL


@pytest.mark.parametrize("layout,gate", [(lib.LAYOUT_QWEN_GATE_UP_MXFP4, lib.SHARED_SIGMOID_GATE),
                                         (lib.LAYOUT_DS_W13_MXFP4, lib.SHARED_ONE)])
def test_decode_forward_with_shared_expert(eng, layout, gate):
    lw = layer(layout, seed=41, gate=gate)
    T, K = 24, 8
    x = synth.activations(T, H, torch.Generator(device=DEV).manual_seed(42), DEV)
    out, (w, idx) = eng.forward(lw, x, K, return_routes=True)
    eng.sync()
    ref = adapter.from_layer(lw).forward(adapter.bits(x), idx.cpu().numpy(), w.cpu().numpy())
    assert rel(adapter.bits(out), ref) <= TOL
