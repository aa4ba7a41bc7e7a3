"""The block-scaled tcgen05 decode kernel (the default for MXFP4 decode calls)
against the CPU oracle and against the register-direct decode kernel
(WM_FLAG_MMA_DECODE; needs a B200).

Weights enter the MMA as E2M1 with their E8M0 scales (exact); token rows as
two E4M3 parts (within 2^-8 of each element).  Tolerance as everywhere:
max|y - y_ref| / max|y_ref| <= 1e-2 on bf16 outputs, with identical top-k
sets (the router is shared with the other paths)."""
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


def rel(a_bits, b_bits):
    return oracle.max_rel_error(oracle.bf16_to_f32(a_bits), oracle.bf16_to_f32(b_bits))


@pytest.fixture(scope="module")
def config1():
    return synth.config(1, device=DEV, batch=64)


def _engines(T, H, I, E, K):
    bs = Engine(0, max_tokens=T, hidden=H, inter=I, experts=E, topk=K)
    mma = Engine(0, max_tokens=T, hidden=H, inter=I, experts=E, topk=K, flags=lib.FLAG_MMA_DECODE)
    return bs, mma


@pytest.mark.parametrize("B", [1, 2, 8, 17, 64])
def test_bs_decode_config1_matches_oracle(config1, B):
    """Config-1 layer (Qwen layout, sigmoid-gated shared expert) at several
    batches, two calls in a row; the block-scaled path launches three expert
    kernels (quantise, gate/up, down) where the register-direct path has four."""
    layer = config1.layer
    bs, mma = _engines(64, 2048, 512, 512, 10)
    x = synth.activations(B, 2048, torch.Generator(device=DEV).manual_seed(300 + B), DEV)
    bs.ctx.profile(True)
    out1, (w, idx) = bs.forward(layer, x, 10, return_routes=True)
    bs.sync()
    kernels = bs.ctx.profile_read()
    bs.ctx.profile(False)
    assert "decode_gate_up" in kernels and "act_f16" not in kernels  # the block-scaled path ran
    out2 = bs.forward(layer, x, 10)
    ref_mma = mma.forward(layer, x, 10, routes=(w, idx))
    bs.sync()
    mma.sync()
    assert torch.equal(out1.view(torch.int16), out2.view(torch.int16))
    ref = adapter.from_layer(layer).forward(adapter.bits(x), idx.cpu().numpy(), w.cpu().numpy())
    assert rel(adapter.bits(out1), ref) <= TOL
    assert rel(adapter.bits(out1), adapter.bits(ref_mma)) <= TOL
    bs.ctx.close()
    mma.ctx.close()


@pytest.mark.parametrize("layout,limit", [(lib.LAYOUT_DS_W13_MXFP4, 10.0), (lib.LAYOUT_QWEN_GATE_UP_MXFP4, 0.0)])
@pytest.mark.parametrize("H,I", [(1024, 512), (512, 1024)])
def test_bs_decode_expert_pairs_match_oracle(layout, limit, H, I):
    E, K, T = 24, 4, 40
    g = torch.Generator(device=DEV).manual_seed(H + I + layout)
    w13, s13 = synth.mxfp4_projection(E, 2 * I, H, g, DEV)
    w2, s2 = synth.mxfp4_projection(E, H, I, g, DEV)
    layer = LayerWeights(layout, H, I, E, Projection.stacked(w13, s13), Projection.stacked(w2, s2),
                         swiglu_limit=limit)
    x = synth.activations(T, H, g, DEV)
    idx = torch.stack([torch.randperm(E, generator=g, device=DEV)[:K] for _ in range(T)]).to(torch.int32)
    idx[:20, 0] = 3  # one expert with more than one 16-token tile
    bs, _ = _engines(T, H, I, E, K)
    out = bs.expert_pairs(layer, x, idx)
    bs.sync()
    ref = adapter.from_layer(layer).pairs(adapter.bits(x), idx.cpu().numpy())
    assert rel(adapter.bits(out), ref) <= TOL
    bs.ctx.close()


def test_bs_decode_config4_shape():
    """A decode call at the config-4 layer shape (H=7168, I=2048, 384 DS-layout
    experts, ungated shared expert, sigmoid top-8)."""
    wl = synth.config(4, device=DEV)
    layer = wl.layer
    x = wl.x[:8].contiguous()
    bs = Engine(0, max_tokens=8, hidden=7168, inter=2048, experts=384, topk=8)
    out, (w, idx) = bs.forward(layer, x, 8, return_routes=True)
    bs.sync()
    ii = idx.cpu().numpy()
    experts = sorted(set(ii.reshape(-1).tolist()))
    remap = {e: i for i, e in enumerate(experts)}
    ref = adapter.from_layer(layer, experts=experts).forward(adapter.bits(x), np.vectorize(remap.get)(ii).astype(
        np.int32), w.cpu().numpy())
    assert rel(adapter.bits(out), ref) <= TOL
    bs.ctx.close()
    del wl, layer
    torch.cuda.empty_cache()
