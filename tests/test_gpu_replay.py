"""Engine.replay (a repeated call shape replayed from a CUDA graph) against
Engine.forward: the same kernels on the same inputs, so the outputs must be
equal bit for bit, for device and pinned host tensors, on consecutive calls
with different inputs (the static input block is refilled every call).
"""
import pytest
import torch

from whallm_b200 import lib, synth
from whallm_b200.layout import Projection
from whallm_b200.moe import Engine, LayerWeights, RouterWeights, SharedExpert

pytestmark = pytest.mark.gpu

DEV = "cuda"
E, H, I, K = 64, 1024, 512, 4


def _layer(seed=11):
    g = torch.Generator(device=DEV).manual_seed(seed)
    w13, s13 = synth.mxfp4_projection(E, 2 * I, H, g, DEV, -8, -2)
    w2, s2 = synth.mxfp4_projection(E, H, I, g, DEV, -8, -2)
    a, b = synth.mxfp4_projection(1, 2 * I, H, g, DEV, -8, -2)
    c, d = synth.mxfp4_projection(1, H, I, g, DEV, -8, -2)
    gw = (torch.randn((H,), generator=g, device=DEV) / H ** 0.5).to(torch.bfloat16)
    shared = SharedExpert(Projection.stacked(a, b), Projection.stacked(c, d), lib.SHARED_SIGMOID_GATE, gw)
    wr = (torch.randn((E, H), generator=g, device=DEV) / H ** 0.5).to(torch.bfloat16)
    return LayerWeights(lib.LAYOUT_QWEN_GATE_UP_MXFP4, H, I, E, Projection.stacked(w13, s13),
                        Projection.stacked(w2, s2), shared=shared, router=RouterWeights(wr, lib.ROUTER_SOFTMAX))


@pytest.mark.parametrize("T", [1, 8, 64])
def test_replay_equals_forward(T):
    eng = Engine(0, max_tokens=256, hidden=H, inter=I, experts=E, topk=K)
    layer = _layer()
    g = torch.Generator(device=DEV).manual_seed(100 + T)
    for step in range(3):
        x = torch.randn((T, H), generator=g, device=DEV).to(torch.bfloat16)
        want = eng.forward(layer, x, K)
        got = eng.replay(layer, x, K)
        torch.cuda.synchronize()
        assert torch.equal(got, want), f"device tensors, step {step}"
        xh = x.cpu().pin_memory()
        oh = torch.empty((T, H), dtype=torch.bfloat16).pin_memory()
        eng.replay(layer, xh, K, out=oh)
        torch.cuda.synchronize()
        assert torch.equal(oh, want.cpu()), f"pinned host tensors, step {step}"
    eng.sync()
    assert len(eng._replays) == 1
    eng.release_replays()


def test_replay_rejects_wrong_shape_and_skips_empty_calls():
    eng = Engine(0, max_tokens=64, hidden=H, inter=I, experts=E, topk=K)
    layer = _layer()
    with pytest.raises(ValueError):
        eng.replay(layer, torch.zeros((4, H + 8), dtype=torch.bfloat16, device=DEV), K)
    assert eng.replay(layer, torch.zeros((0, H), dtype=torch.bfloat16, device=DEV), K).shape == (0, H)
    assert not getattr(eng, "_replays", {})
