"""WM_FLAG_FUSED_DECODE: the block-scaled decode path's gate/up and down
kernels as one persistent launch (needs a B200).

The launch runs the same items, MMAs and epilogues as the two kernels, so
its outputs must equal theirs bit for bit, on consecutive calls of different
sizes (the per-tile counts the down items wait on are cleared by the launch
itself for the next one), and stay within the oracle's tolerance.  Off by
default and not yet run on a GPU: these tests run only with
WM_RUN_FUSED_DECODE_TESTS=1."""
import os

import pytest
import torch

import oracle
from oracle import adapter
from whallm_b200 import lib, synth
from whallm_b200.moe import Engine

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(os.environ.get("WM_RUN_FUSED_DECODE_TESTS") != "1",
                                 reason="the one-launch decode has not been run on a GPU yet")]
TOL = 1e-2
DEV = "cuda"


def test_fused_decode_matches_two_launches_on_consecutive_calls():
    wl = synth.config(1, device=DEV, batch=64)
    layer, K = wl.layer, wl.K
    fused = Engine(0, max_tokens=64, hidden=2048, inter=512, experts=512, topk=K, flags=lib.FLAG_FUSED_DECODE)
    two = Engine(0, max_tokens=64, hidden=2048, inter=512, experts=512, topk=K)
    for call, B in enumerate([64, 8, 1, 64, 17]):
        x = synth.activations(B, 2048, torch.Generator(device=DEV).manual_seed(700 + call), DEV)
        fused.ctx.profile(True)
        fused.ctx.profile_reset()
        got, (w, idx) = fused.forward(layer, x, K, return_routes=True)
        fused.sync()
        kernels = fused.ctx.profile_read()
        fused.ctx.profile(False)
        assert "decode_fused" in kernels and "decode_gate_up" not in kernels
        want = two.forward(layer, x, K, routes=(w, idx))
        two.sync()
        assert torch.equal(got.view(torch.int16), want.view(torch.int16)), f"call {call}, batch {B}"
    ref = adapter.from_layer(layer).forward(adapter.bits(x), idx.cpu().numpy(), w.cpu().numpy())
    err = oracle.max_rel_error(oracle.bf16_to_f32(adapter.bits(got)), oracle.bf16_to_f32(ref))
    assert err <= TOL
    fused.ctx.close()
    two.ctx.close()


@pytest.mark.parametrize("layout,limit,H,I", [(lib.LAYOUT_DS_W13_MXFP4, 10.0, 1024, 512),
                                              (lib.LAYOUT_QWEN_GATE_UP_MXFP4, 0.0, 512, 1024)])
def test_fused_decode_expert_pairs_shapes(layout, limit, H, I):
    """Other shapes and the up-first layout with the clamp: the routed rows of
    the one launch equal the two kernels' and the oracle's."""
    from whallm_b200.layout import Projection
    from whallm_b200.moe import LayerWeights
    E, K, T = 24, 4, 40
    g = torch.Generator(device=DEV).manual_seed(H + I + layout)
    w13, s13 = synth.mxfp4_projection(E, 2 * I, H, g, DEV)
    w2, s2 = synth.mxfp4_projection(E, H, I, g, DEV)
    layer = LayerWeights(layout, H, I, E, Projection.stacked(w13, s13), Projection.stacked(w2, s2),
                         swiglu_limit=limit)
    x = synth.activations(T, H, g, DEV)
    idx = torch.stack([torch.randperm(E, generator=g, device=DEV)[:K] for _ in range(T)]).to(torch.int32)
    idx[:20, 0] = 3  # one expert with more than one 16-token tile
    fused = Engine(0, max_tokens=T, hidden=H, inter=I, experts=E, topk=K, flags=lib.FLAG_FUSED_DECODE)
    two = Engine(0, max_tokens=T, hidden=H, inter=I, experts=E, topk=K)
    for _ in range(2):
        got = fused.expert_pairs(layer, x, idx)
        want = two.expert_pairs(layer, x, idx)
        torch.cuda.synchronize()
        assert torch.equal(got.view(torch.int16), want.view(torch.int16))
    ref = adapter.from_layer(layer).pairs(adapter.bits(x), idx.cpu().numpy())
    err = oracle.max_rel_error(oracle.bf16_to_f32(adapter.bits(got)), oracle.bf16_to_f32(ref))
    assert err <= TOL
    fused.ctx.close()
    two.ctx.close()
