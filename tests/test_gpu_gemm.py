"""The tcgen05 grouped-GEMM (prefill) paths vs the CPU oracle (needs a B200): the
block-scaled GEMM for the full-size MXFP4 configs, the kind::f16 GEMM for the
small shapes and FP8.

Same tolerance as the decode path: max|y - y_ref| / max|y_ref| <= 1e-2 on bf16
outputs.  Full-size layers are checked on sampled tokens (the oracle runs only
the experts those tokens reach) plus whole-output properties.
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


def rel(y_bits, ref_bits):
    return oracle.max_rel_error(oracle.bf16_to_f32(y_bits), oracle.bf16_to_f32(ref_bits))


def small_layer(layout, E, H, I, seed, gate=lib.SHARED_NONE, limit=0.0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    proj = synth.projection_for(layout)
    w13, s13 = proj(E, 2 * I, H, g, DEV)
    w2, s2 = proj(E, H, I, g, DEV)
    shared = None
    if gate != lib.SHARED_NONE:
        a, b = proj(1, 2 * I, H, g, DEV)
        c, d = proj(1, H, I, g, DEV)
        gw = (torch.randn((H,), generator=g, device=DEV) / H ** 0.5).to(torch.bfloat16)
        shared = SharedExpert(Projection.stacked(a, b), Projection.stacked(c, d), gate,
                              gw if gate == lib.SHARED_SIGMOID_GATE else None)
    wr = (torch.randn((E, H), generator=g, device=DEV) / H ** 0.5).to(torch.bfloat16)
    return LayerWeights(layout, H, I, E, Projection.stacked(w13, s13), Projection.stacked(w2, s2), shared=shared,
                        router=RouterWeights(wr, lib.ROUTER_SOFTMAX), swiglu_limit=limit)


@pytest.fixture(scope="module")
def gemm_engine():
    eng = Engine(0, max_tokens=1024, hidden=1024, inter=512, experts=16, topk=8, gemv_max_tokens=-1)
    yield eng
    eng.ctx.close()


@pytest.fixture(scope="module")
def gemv_engine():
    eng = Engine(0, max_tokens=1024, hidden=1024, inter=512, experts=16, topk=8, gemv_max_tokens=100000)
    yield eng
    eng.ctx.close()


def test_gemm_single_tile(gemm_engine):
    """One expert, one 128-row tile: the smallest grouped GEMM."""
    layer = small_layer(lib.LAYOUT_QWEN_GATE_UP_MXFP4, 1, 256, 128, seed=1)
    x = synth.activations(100, 256, torch.Generator(device=DEV).manual_seed(2), DEV)
    idx = torch.zeros((100, 1), dtype=torch.int32, device=DEV)
    out = gemm_engine.expert_pairs(layer, x, idx)
    gemm_engine.sync()
    assert gemm_engine.ctx.counters().gemm_calls >= 1
    ref = adapter.from_layer(layer).pairs(adapter.bits(x), idx.cpu().numpy())
    assert rel(adapter.bits(out), ref) <= TOL


@pytest.mark.parametrize("layout,limit", [(lib.LAYOUT_QWEN_GATE_UP_MXFP4, 0.0), (lib.LAYOUT_DS_W13_MXFP4, 10.0),
                                          (lib.LAYOUT_W13_FP8_B128, 0.0), (lib.LAYOUT_W13_FP8_B32, 0.0)])
@pytest.mark.parametrize("T", [1, 65, 300])
def test_gemm_expert_pairs_match_oracle(gemm_engine, layout, limit, T):
    E, H, I, K = 16, 512, 256, 4
    layer = small_layer(layout, E, H, I, seed=10 + layout, limit=limit)
    g = torch.Generator(device=DEV).manual_seed(20 + T)
    x = synth.activations(T, H, g, DEV)
    idx = torch.stack([torch.randperm(E, generator=g, device=DEV)[:K] for _ in range(T)]).to(torch.int32)
    out = gemm_engine.expert_pairs(layer, x, idx)
    gemm_engine.sync()
    ref = adapter.from_layer(layer).pairs(adapter.bits(x), idx.cpu().numpy())
    assert rel(adapter.bits(out), ref) <= TOL


@pytest.mark.parametrize("layout,gate", [(lib.LAYOUT_QWEN_GATE_UP_MXFP4, lib.SHARED_SIGMOID_GATE),
                                         (lib.LAYOUT_W13_FP8_B128, lib.SHARED_ONE),
                                         (lib.LAYOUT_W13_FP8_B32, lib.SHARED_ONE)])
def test_gemm_forward_matches_gemv_and_oracle(gemm_engine, gemv_engine, layout, gate):
    E, H, I, K, T = 16, 1024, 512, 8, 257
    layer = small_layer(layout, E, H, I, seed=30 + layout, gate=gate)
    x = synth.activations(T, H, torch.Generator(device=DEV).manual_seed(31), DEV)
    out_a, (w, idx) = gemm_engine.forward(layer, x, K, return_routes=True)
    out_b = gemv_engine.forward(layer, x, K, routes=(w, idx))
    gemm_engine.sync()
    gemv_engine.sync()
    assert rel(adapter.bits(out_a), adapter.bits(out_b)) <= TOL
    ref = adapter.from_layer(layer).forward(adapter.bits(x), idx.cpu().numpy(), w.cpu().numpy())
    assert rel(adapter.bits(out_a), ref) <= TOL


def _check_sampled(layer, x, out, w, idx, tokens):
    """Oracle on `tokens` only, over the experts they reach (remapped)."""
    ii = idx.cpu().numpy()[tokens]
    ww = w.cpu().numpy()[tokens]
    experts = sorted(set(ii.reshape(-1).tolist()))
    remap = {e: i for i, e in enumerate(experts)}
    sub_idx = np.vectorize(remap.get)(ii).astype(np.int32)
    ref = adapter.from_layer(layer, experts=experts).forward(adapter.bits(x[tokens]), sub_idx, ww)
    got = adapter.bits(out[tokens])
    return rel(got, ref)


def _coverage_sample(idx: torch.Tensor, E: int, rng: np.random.Generator, n_random: int, tile: int = 128,
                     groups: int = 0) -> np.ndarray:
    """Tokens for a sampled oracle check of a full-size call: random ones plus
    the tokens that reach the most popular expert (its last one included), the
    last token of experts whose rows end in a partial 128-row tile (the sorted
    rows keep (token, k) order, so an expert's last token owns its last row),
    the first and last token (the shared expert's first and last rows) and,
    with `groups`, tokens reaching every expert group."""
    ii = idx.cpu().numpy()
    T = ii.shape[0]
    counts = np.bincount(ii.reshape(-1), minlength=E)
    head = int(counts.argmax())
    head_tokens = np.flatnonzero((ii == head).any(axis=1))
    picks = set(rng.choice(T, n_random, replace=False).tolist())
    picks.update(head_tokens[:: max(1, head_tokens.size // 7)][:7].tolist())
    picks.add(int(head_tokens[-1]))
    partial = [e for e in np.argsort(-counts) if counts[e] % tile and counts[e] > tile][:8]
    partial += [e for e in np.argsort(counts) if 0 < counts[e] < tile][:4]
    for e in partial:
        picks.add(int(np.flatnonzero((ii == e).any(axis=1))[-1]))
    picks.update((0, T - 1))
    if groups:
        size = E // groups
        for g_ in range(groups):
            hit = np.flatnonzero(((ii // size) == g_).any(axis=1))
            picks.update(hit[:2].tolist())
    return np.array(sorted(picks), dtype=np.int64)


def test_config2_prefill_full_size():
    wl = synth.config(2, device=DEV)
    eng = Engine(0, max_tokens=16384, hidden=2048, inter=512, experts=512, topk=10)
    out, (w, idx) = eng.forward(wl.layer, wl.x, wl.K, return_routes=True)
    eng.sync()
    assert eng.ctx.counters().gemm_calls == 1 and eng.ctx.counters().bs_gemm_calls == 1
    assert torch.isfinite(out.float()).all()
    counts = torch.bincount(idx.reshape(-1).long(), minlength=512)
    assert counts.sum().item() == 16384 * 10 and counts.max().item() > 20 * counts.float().median().item()
    tokens = _coverage_sample(idx, 512, np.random.default_rng(0), 60)
    assert tokens.size >= 64
    assert _check_sampled(wl.layer, wl.x, out, w, idx, tokens) <= TOL
    eng.ctx.close()


def test_config3_fp8_full_size():
    wl = synth.config(3, device=DEV)
    eng = Engine(0, max_tokens=8192, hidden=7168, inter=2048, experts=256, topk=8)
    out, (w, idx) = eng.forward(wl.layer, wl.x, wl.K, return_routes=True)
    eng.sync()
    assert torch.isfinite(out.float()).all()
    # group-limited routing: every token's experts lie in at most 4 of the 8 groups
    groups = (idx.long() // 32)
    per_token = [torch.unique(r).numel() for r in groups[:256]]
    assert max(per_token) <= 4
    tokens = _coverage_sample(idx, 256, np.random.default_rng(1), 50, groups=8)
    assert tokens.size >= 64
    hit_groups = set((idx.cpu().numpy()[tokens] // 32).reshape(-1).tolist())
    assert hit_groups == set(range(8))
    assert _check_sampled(wl.layer, wl.x, out, w, idx, tokens) <= TOL
    eng.ctx.close()
    del wl, eng
    torch.cuda.empty_cache()


def test_config4_layer_full_size():
    """One layer of the config-4 stack at its shape -- H=7168, 384 MXFP4
    experts of I=2048 (w13 = [w3; w1]), ungated shared expert, sigmoid top-8,
    256 decode + 4096 prefill tokens in one call (grouped GEMM) -- against the
    oracle on sampled tokens, with the routes checked against the oracle
    router; then a decode-sized call of 8 tokens (decode kernels)."""
    wl = synth.config(4, device=DEV)
    layer = wl.layer
    T = wl.x.shape[0]
    eng = Engine(0, max_tokens=T, hidden=7168, inter=2048, experts=384, topk=8)
    out, (w, idx) = eng.forward(layer, wl.x, wl.K, return_routes=True)
    eng.sync()
    assert eng.ctx.counters().gemm_calls == 1 and eng.ctx.counters().bs_gemm_calls == 1
    assert torch.isfinite(out.float()).all()
    tokens = _coverage_sample(idx, 384, np.random.default_rng(2), 16)
    tokens = np.union1d(tokens, np.array([1, 100, 255, 256, 257], dtype=np.int64))  # decode / prefill boundary
    logits = oracle.router_logits(adapter.bits(wl.x[tokens]), adapter.bits(layer.router.weight))
    want_idx, _ = oracle.route(oracle.ROUTER_SIGMOID, logits, wl.K)
    got_idx = idx.cpu().numpy()[tokens]
    assert [set(r) for r in got_idx.tolist()] == [set(r) for r in want_idx.tolist()]
    assert _check_sampled(layer, wl.x, out, w, idx, tokens) <= TOL
    # decode-sized call at this shape
    xd = wl.x[:8].contiguous()
    outd, (wd, idd) = eng.forward(layer, xd, wl.K, return_routes=True)
    eng.sync()
    assert eng.ctx.counters().gemm_calls == 1  # the short call took the decode kernels
    assert _check_sampled(layer, xd, outd, wd, idd, np.arange(8)) <= TOL
    eng.ctx.close()
    del wl, layer, eng
    torch.cuda.empty_cache()
