"""Calls of up to 64 tokens on the block-scaled decode path: the plan and the
token images in one launch, and for router calls of up to 4 tokens the top-k
in that launch too (needs a B200).

The one launch must give the same bits as the launches it replaces (top-k,
plan, quantise; WM_FLAG_SPLIT_SMALL_CALLS keeps them): identical routes
(indices and weights) and identical layer outputs, for every router kind,
with and without the shared expert and the pre-MoE norm, and for given
routes.  One case per router kind is also checked against the CPU oracle
(max|y - y_ref| / max|y_ref| <= 1e-2, identical top-k sets)."""
import pytest
import torch

import oracle
from oracle import adapter
from whallm_b200 import lib, synth
from whallm_b200.layout import Projection
from whallm_b200.moe import Engine, LayerWeights, PreNorm, RouterWeights, SharedExpert

pytestmark = pytest.mark.gpu
TOL = 1e-2
DEV = "cuda"
FLAG_SPLIT = lib.FLAG_SPLIT_SMALL_CALLS


def _layer(E, H, I, kind, shared, norm, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
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
    bias = None
    groups, keep = 1, 1
    if kind != lib.ROUTER_SOFTMAX:
        bias = 0.1 * torch.randn((E,), generator=g, device=DEV)
    if kind == lib.ROUTER_SIGMOID_GROUPED:
        groups, keep = 8, 4
    router = RouterWeights(wr, kind, bias, groups, keep, 2.5 if kind != lib.ROUTER_SOFTMAX else 1.0)
    pre = None
    if norm:
        pre = PreNorm((1.0 + 0.2 * torch.randn((H,), generator=g, device=DEV)).to(torch.bfloat16), 1e-6)
    return LayerWeights(lib.LAYOUT_QWEN_GATE_UP_MXFP4 if kind == lib.ROUTER_SOFTMAX else lib.LAYOUT_DS_W13_MXFP4,
                        H, I, E, Projection.stacked(w13, s13), Projection.stacked(w2, s2), shared=sh, router=router,
                        swiglu_limit=0.0 if kind == lib.ROUTER_SOFTMAX else 10.0, norm=pre)


def _run(eng, layer, x, K):
    """Output, routes, the kernels that ran and the normalised rows (or x)."""
    xn = torch.empty_like(x) if layer.norm is not None else None
    eng.ctx.profile(True)
    eng.ctx.profile_reset()
    out, (w, idx) = eng.forward(layer, x, K, return_routes=True, x_norm=xn)
    eng.sync()
    kernels = eng.ctx.profile_read()
    eng.ctx.profile(False)
    return out, w, idx, kernels, (x if xn is None else xn)


CASES = [
    # kind, E, K, shared, norm
    (lib.ROUTER_SOFTMAX, 512, 10, lib.SHARED_SIGMOID_GATE, False),
    (lib.ROUTER_SOFTMAX, 256, 8, lib.SHARED_NONE, True),
    (lib.ROUTER_SQRTSOFTPLUS, 256, 6, lib.SHARED_ONE, False),
    (lib.ROUTER_SIGMOID, 512, 8, lib.SHARED_SIGMOID_GATE, True),
    (lib.ROUTER_SIGMOID_GROUPED, 256, 8, lib.SHARED_ONE, False),
]


@pytest.mark.parametrize("kind,E,K,shared,norm", CASES)
@pytest.mark.parametrize("T", [1, 3, 4])
def test_one_launch_matches_three_launches_bit_for_bit(kind, E, K, shared, norm, T):
    H, I = 1024, 512
    layer = _layer(E, H, I, kind, shared, norm, seed=1000 + 10 * kind + E + K)
    x = synth.activations(T, H, torch.Generator(device=DEV).manual_seed(77 + T), DEV)
    one = Engine(0, max_tokens=16, hidden=H, inter=I, experts=E, topk=K)
    three = Engine(0, max_tokens=16, hidden=H, inter=I, experts=E, topk=K, flags=FLAG_SPLIT)
    o1, w1, i1, k1, xin = _run(one, layer, x, K)
    o3, w3, i3, k3, _ = _run(three, layer, x, K)
    # the group-limited router keeps its own top-k launch; the others select inside the one launch
    selects = kind != lib.ROUTER_SIGMOID_GROUPED
    assert "route_plan_quant" in k1 and ("router_topk" in k1) != selects and "plan" not in k1
    assert "gather_rows" not in k1
    assert "route_plan_quant" not in k3 and "router_topk" in k3 and "plan" in k3
    assert torch.equal(i1, i3)
    assert torch.equal(w1.view(torch.int32), w3.view(torch.int32))
    assert torch.equal(o1.view(torch.int16), o3.view(torch.int16))
    # a second call on the same handle (workspace reused) gives the same bits
    o1b = one.forward(layer, x, K)
    one.sync()
    assert torch.equal(o1.view(torch.int16), o1b.view(torch.int16))
    if T == 3:
        r = layer.router
        logits = oracle.router_logits(adapter.bits(xin), adapter.bits(r.weight))
        bias = None if r.bias is None else r.bias.cpu().numpy()
        want, _ = oracle.route(kind, logits, K, bias, r.n_groups, r.topk_groups, r.route_scale)
        assert [set(v) for v in i1.cpu().numpy().tolist()] == [set(v) for v in want.tolist()]
        ref = adapter.from_layer(layer).forward(adapter.bits(xin), i1.cpu().numpy(), w1.cpu().numpy())
        err = oracle.max_rel_error(oracle.bf16_to_f32(adapter.bits(o1)), oracle.bf16_to_f32(ref))
        assert err <= TOL
    one.ctx.close()
    three.ctx.close()


@pytest.mark.parametrize("B", [1, 4])
def test_config1_small_batches_replayed_match_three_launches(B):
    """The config-1 layer (H 2048, 512 experts of I 512 + shared, top-10) at
    batch 1 and 4 through Engine.replay (a captured CUDA graph): the same
    bits as the three-launch path, and within the tolerance of the oracle."""
    wl = synth.config(1, device=DEV, batch=B)
    layer, K = wl.layer, wl.K
    one = Engine(0, max_tokens=64, hidden=2048, inter=512, experts=512, topk=K)
    three = Engine(0, max_tokens=64, hidden=2048, inter=512, experts=512, topk=K, flags=FLAG_SPLIT)
    for call in range(3):
        x = synth.activations(B, 2048, torch.Generator(device=DEV).manual_seed(900 + call), DEV)
        got = one.replay(layer, x, K)
        want, (w, idx) = three.forward(layer, x, K, return_routes=True)
        torch.cuda.synchronize()
        assert torch.equal(got.view(torch.int16), want.view(torch.int16))
    ref = adapter.from_layer(layer).forward(adapter.bits(x), idx.cpu().numpy(), w.cpu().numpy())
    err = oracle.max_rel_error(oracle.bf16_to_f32(adapter.bits(got)), oracle.bf16_to_f32(ref))
    assert err <= TOL
    one.ctx.close()
    three.ctx.close()


@pytest.mark.parametrize("kind,E,K,shared,norm", CASES[:1] + CASES[3:])
@pytest.mark.parametrize("T", [5, 17, 64])
def test_plan_and_images_in_one_launch_match_the_two_launches(kind, E, K, shared, norm, T):
    """5 to 64 tokens: the top-k kernel, then the plan and the token images in
    one launch -- the same bits as the plan and quantise kernels."""
    H, I = 1024, 512
    layer = _layer(E, H, I, kind, shared, norm, seed=2000 + 10 * kind + E + K)
    x = synth.activations(T, H, torch.Generator(device=DEV).manual_seed(55 + T), DEV)
    one = Engine(0, max_tokens=64, hidden=H, inter=I, experts=E, topk=K)
    two = Engine(0, max_tokens=64, hidden=H, inter=I, experts=E, topk=K, flags=FLAG_SPLIT)
    o1, w1, i1, k1, _ = _run(one, layer, x, K)
    o2, w2, i2, k2, _ = _run(two, layer, x, K)
    assert "route_plan_quant" in k1 and "router_topk" in k1 and "plan" not in k1 and "gather_rows" not in k1
    assert "route_plan_quant" not in k2 and "plan" in k2 and "gather_rows" in k2
    assert torch.equal(i1, i2) and torch.equal(w1.view(torch.int32), w2.view(torch.int32))
    assert torch.equal(o1.view(torch.int16), o2.view(torch.int16))
    one.ctx.close()
    two.ctx.close()


@pytest.mark.parametrize("T,K,E", [(64, 10, 512), (40, 8, 256), (3, 16, 64)])
def test_given_routes_in_one_launch_match_the_two_launches(T, K, E):
    """Caller-given routes (no router), an expert named by many tokens and by
    none: the same bits as the plan and quantise kernels, and the oracle."""
    H, I = 1024, 512
    layer = _layer(E, H, I, lib.ROUTER_SOFTMAX, lib.SHARED_SIGMOID_GATE, False, seed=3000 + T)
    g = torch.Generator(device=DEV).manual_seed(4000 + T)
    x = synth.activations(T, H, g, DEV)
    idx = torch.stack([torch.randperm(E, generator=g, device=DEV)[:K] for _ in range(T)]).to(torch.int32)
    idx[:, 0] = 3  # every token names expert 3 (more than one 16-row tile at T > 16)
    idx[:, 1] = torch.where(idx[:, 1] == 3, torch.full_like(idx[:, 1], 5), idx[:, 1])
    w = torch.rand((T, K), generator=g, device=DEV)
    one = Engine(0, max_tokens=64, hidden=H, inter=I, experts=E, topk=K)
    two = Engine(0, max_tokens=64, hidden=H, inter=I, experts=E, topk=K, flags=FLAG_SPLIT)
    got = one.forward(layer, x, K, routes=(w, idx))
    want = two.forward(layer, x, K, routes=(w, idx))
    one.sync()
    two.sync()
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))
    ref = adapter.from_layer(layer).forward(adapter.bits(x), idx.cpu().numpy(), w.cpu().numpy())
    err = oracle.max_rel_error(oracle.bf16_to_f32(adapter.bits(got)), oracle.bf16_to_f32(ref))
    assert err <= TOL
    one.ctx.close()
    two.ctx.close()


@pytest.mark.parametrize("kind", [lib.ROUTER_SOFTMAX, lib.ROUTER_SQRTSOFTPLUS, lib.ROUTER_SIGMOID])
@pytest.mark.parametrize("E,K", [(512, 10), (384, 8), (1024, 16), (256, 32), (128, 6)])
def test_group_topk_of_short_calls_matches_the_one_warp_topk(kind, E, K):
    """Calls of up to 4 tokens select with four warps per token; longer calls
    with one warp per token.  The first 4 tokens of a 100-token call (one warp
    per token, the same logits) must get the same routes, bit for bit, as the
    same 4 tokens routed alone, and the oracle's selection on those logits."""
    import numpy as np
    H = 512
    g = torch.Generator(device=DEV).manual_seed(6000 + E + K + kind)
    w13, s13 = synth.mxfp4_projection(8, 128, H, g, DEV)
    w2, s2 = synth.mxfp4_projection(8, H, 64, g, DEV)
    wr = (torch.randn((E, H), generator=g, device=DEV) / H ** 0.5).to(torch.bfloat16)
    bias = None if kind == lib.ROUTER_SOFTMAX else (0.1 * torch.randn((E,), generator=g, device=DEV))
    layer = LayerWeights(lib.LAYOUT_QWEN_GATE_UP_MXFP4, H, 64, E, Projection.stacked(w13, s13),
                         Projection.stacked(w2, s2), router=RouterWeights(wr, kind, bias, 1, 1, 1.5))
    x = synth.activations(100, H, g, DEV)
    eng = Engine(0, max_tokens=128, hidden=H, inter=64, experts=E, topk=K)
    w_long, i_long, logits = eng.route(layer, x, K, with_logits=True)
    w_short, i_short = eng.route(layer, x[:4].contiguous(), K)
    eng.sync()
    assert torch.equal(i_short, i_long[:4])
    assert torch.equal(w_short.view(torch.int32), w_long[:4].view(torch.int32))
    bn = None if bias is None else bias.cpu().numpy()
    oi, ow = oracle.route(kind, logits.cpu().numpy(), K, bn, 1, 1, 1.5)
    np.testing.assert_array_equal(i_long.cpu().numpy(), oi)
    np.testing.assert_allclose(w_long.cpu().numpy(), ow, rtol=1e-5, atol=1e-7)
    eng.ctx.close()
