"""wm_moe_forward_noalloc: the allocation-free decode entry point (needs a B200).

Some callers cannot call cudaMalloc -- for example a serving process whose GPU
memory is fixed at start-up, or a host framework that owns all device memory
through its own allocator.  This entry point runs the decode MoE block with
its scratch in a static device array instead of a handle's workspace.  The
test calls it through the C ABI twice in a row and checks both results against
the regular wm_moe_forward on the same inputs, within the tolerance of the
other parity tests (max|y - y_ref| / max|y_ref| <= 1e-2).  This file is named
so that pytest collects it last.
"""
import ctypes

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


def _layer(E=16, H=512, I=256, seed=7):
    g = torch.Generator(device=DEV).manual_seed(seed)
    w13, s13 = synth.mxfp4_projection(E, 2 * I, H, g, DEV)
    w2, s2 = synth.mxfp4_projection(E, H, I, g, DEV)
    a, b = synth.mxfp4_projection(1, 2 * I, H, g, DEV)
    c, d = synth.mxfp4_projection(1, H, I, g, DEV)
    gate = (torch.randn((H,), generator=g, device=DEV) / H ** 0.5).to(torch.bfloat16)
    wr = (torch.randn((E, H), generator=g, device=DEV) / H ** 0.5).to(torch.bfloat16)
    return LayerWeights(lib.LAYOUT_QWEN_GATE_UP_MXFP4, H, I, E, Projection.stacked(w13, s13),
                        Projection.stacked(w2, s2),
                        shared=SharedExpert(Projection.stacked(a, b), Projection.stacked(c, d),
                                            lib.SHARED_SIGMOID_GATE, gate),
                        router=RouterWeights(wr, lib.ROUTER_SOFTMAX))


def _noalloc(eng: Engine, layer: LayerWeights, x: torch.Tensor, K: int, out: torch.Tensor):
    a = eng._args(layer, x, K)
    eng._with_shared(a, layer)
    eng._with_router(a, layer.router)
    a.out = out.data_ptr()
    err = ctypes.create_string_buffer(256)
    rc = lib.load().wm_moe_forward_noalloc(ctypes.byref(a), torch.cuda.current_stream().cuda_stream, err, len(err))
    return rc, err.value.decode()


def test_noalloc_matches_wm_moe_forward_twice():
    layer = _layer()
    K, T = 4, 8
    eng = Engine(0, max_tokens=64, hidden=512, inter=256, experts=16, topk=K)
    x = synth.activations(T, 512, torch.Generator(device=DEV).manual_seed(8), DEV)
    ref = eng.forward(layer, x, K)
    eng.sync()
    for _ in range(2):
        out = torch.full((T, 512), float("nan"), dtype=torch.bfloat16, device=DEV)
        rc, msg = _noalloc(eng, layer, x, K, out)
        assert rc == lib.WM_OK, msg
        torch.cuda.synchronize()
        err = oracle.max_rel_error(oracle.bf16_to_f32(adapter.bits(out)), oracle.bf16_to_f32(adapter.bits(ref)))
        assert err <= TOL
    eng.ctx.close()


def _status():
    err = ctypes.create_string_buffer(256)
    rc = lib.load().wm_moe_forward_noalloc_status(torch.cuda.current_stream().cuda_stream, err, len(err))
    return rc, err.value.decode()


@pytest.mark.parametrize("B", [1, 8])
def test_noalloc_config1_decode_matches_oracle(B):
    """The config-1 decode layer (H=2048, 512 experts of I=512 + shared, top-10
    softmax) at batch 1 and 8: two calls in a row, each against the CPU
    oracle on the routes the call chose, and no device error recorded."""
    wl = synth.config(1, device=DEV, batch=B)
    layer, K = wl.layer, wl.K
    eng = Engine(0, max_tokens=64, hidden=2048, inter=512, experts=512, topk=K)
    layer_np = adapter.from_layer(layer)
    for call in range(2):
        x = synth.activations(B, 2048, torch.Generator(device=DEV).manual_seed(40 + call), DEV)
        out = torch.full((B, 2048), float("nan"), dtype=torch.bfloat16, device=DEV)
        ri = torch.empty((B, K), dtype=torch.int32, device=DEV)
        rw = torch.empty((B, K), dtype=torch.float32, device=DEV)
        a = eng._args(layer, x, K)
        eng._with_shared(a, layer)
        eng._with_router(a, layer.router)
        a.out, a.out_idx, a.out_w = out.data_ptr(), ri.data_ptr(), rw.data_ptr()
        err = ctypes.create_string_buffer(256)
        rc = lib.load().wm_moe_forward_noalloc(ctypes.byref(a), torch.cuda.current_stream().cuda_stream, err,
                                               len(err))
        assert rc == lib.WM_OK, err.value.decode()
        rc, msg = _status()
        assert rc == lib.WM_OK, msg
        logits = oracle.router_logits(adapter.bits(x), adapter.bits(layer.router.weight))
        want_idx, _ = oracle.route(oracle.ROUTER_SOFTMAX, logits, K)
        assert [set(r) for r in ri.cpu().numpy().tolist()] == [set(r) for r in want_idx.tolist()]
        ref = layer_np.forward(adapter.bits(x), ri.cpu().numpy(), rw.cpu().numpy())
        e = oracle.max_rel_error(oracle.bf16_to_f32(adapter.bits(out)), oracle.bf16_to_f32(ref))
        assert e <= TOL
    eng.ctx.close()


def test_noalloc_reports_out_of_range_routes():
    """A caller-given route naming an expert outside [0, E) is recorded on the
    device: the status accessor reports it, the bad route adds nothing to its
    token, and the next clean call clears the record."""
    layer = _layer()
    K, T, E = 4, 8, 16
    eng = Engine(0, max_tokens=64, hidden=512, inter=256, experts=E, topk=K)
    g = torch.Generator(device=DEV).manual_seed(50)
    x = synth.activations(T, 512, g, DEV)
    idx = torch.stack([torch.randperm(E, generator=g, device=DEV)[:K] for _ in range(T)]).to(torch.int32)
    w = torch.rand((T, K), generator=g, device=DEV)
    bad = idx.clone()
    bad[3, 2] = E + 5  # out of range
    w_bad = w.clone()

    def call(routes_idx, routes_w):
        out = torch.empty((T, 512), dtype=torch.bfloat16, device=DEV)
        a = eng._args(layer, x, K)
        eng._with_shared(a, layer)
        a.routes_idx, a.routes_w, a.out = routes_idx.data_ptr(), routes_w.data_ptr(), out.data_ptr()
        err = ctypes.create_string_buffer(256)
        rc = lib.load().wm_moe_forward_noalloc(ctypes.byref(a), torch.cuda.current_stream().cuda_stream, err,
                                               len(err))
        assert rc == lib.WM_OK, err.value.decode()
        return out

    out = call(bad, w_bad)
    rc, msg = _status()
    assert rc == lib.WM_ERROR and "outside the model" in msg, msg
    # the bad pair contributes nothing: the same as a zero weight on an in-range expert
    w_zero = w.clone()
    w_zero[3, 2] = 0.0
    want = eng.forward(layer, x, K, routes=(w_zero, idx))
    eng.sync()
    e = oracle.max_rel_error(oracle.bf16_to_f32(adapter.bits(out)), oracle.bf16_to_f32(adapter.bits(want)))
    assert e <= TOL
    call(idx, w)
    rc, msg = _status()
    assert rc == lib.WM_OK, msg
    eng.ctx.close()


def test_noalloc_rejects_sizes_beyond_its_scratch():
    layer = _layer(E=64, H=2048, I=512, seed=9)
    K, T = 8, 1024  # rows (T*K + T) * (H + I) * 2 bytes = 47 MB, beyond the 8 MiB array
    eng = Engine(0, max_tokens=T, hidden=2048, inter=512, experts=64, topk=K)
    x = synth.activations(T, 2048, torch.Generator(device=DEV).manual_seed(10), DEV)
    out = torch.empty((T, 2048), dtype=torch.bfloat16, device=DEV)
    rc, msg = _noalloc(eng, layer, x, K, out)
    assert rc == lib.WM_ERROR and "scratch" in msg
    eng.ctx.close()


@pytest.mark.parametrize("H", [512, 576])  # 512: norm fused into the router; 576: the RMSNorm kernel first
def test_noalloc_with_pre_moe_norm(H):
    """With a norm weight the caller supplies x_norm; the result matches
    wm_moe_forward with the same norm, and x_norm holds the normalised rows."""
    from whallm_b200.moe import PreNorm
    layer = _layer(H=H, seed=11)
    g = torch.Generator(device=DEV).manual_seed(12)
    layer.norm = PreNorm((1.0 + 0.2 * torch.randn((H,), generator=g, device=DEV)).to(torch.bfloat16), 1e-6)
    K, T = 4, 8
    eng = Engine(0, max_tokens=64, hidden=H, inter=256, experts=16, topk=K)
    x = synth.activations(T, H, torch.Generator(device=DEV).manual_seed(13), DEV)
    xn_ref = torch.empty_like(x)
    ref = eng.forward(layer, x, K, x_norm=xn_ref)
    eng.sync()
    out = torch.empty((T, H), dtype=torch.bfloat16, device=DEV)
    xn = torch.empty_like(x)
    a = eng._args(layer, x, K)
    eng._with_shared(a, layer)
    eng._with_router(a, layer.router)
    a.out, a.x_norm = out.data_ptr(), xn.data_ptr()
    err = ctypes.create_string_buffer(256)
    rc = lib.load().wm_moe_forward_noalloc(ctypes.byref(a), torch.cuda.current_stream().cuda_stream, err, len(err))
    assert rc == lib.WM_OK, err.value.decode()
    torch.cuda.synchronize()
    assert torch.equal(xn.view(torch.int16), xn_ref.view(torch.int16))
    e = oracle.max_rel_error(oracle.bf16_to_f32(adapter.bits(out)), oracle.bf16_to_f32(adapter.bits(ref)))
    assert e <= TOL
    a.x_norm = None  # a norm without the caller's rows is refused
    rc = lib.load().wm_moe_forward_noalloc(ctypes.byref(a), torch.cuda.current_stream().cuda_stream, err, len(err))
    assert rc == lib.WM_ERROR and "x_norm" in err.value.decode()
    eng.ctx.close()


def test_small_noalloc_call_keeps_a_larger_handles_limits():
    """Kernel shared-memory limits only ever grow: an allocation-free call with
    a small H after a handle sized for H = 7168 must not lower the GEMV's limit
    that handle's FP8 calls need (CUDA would refuse their launches)."""
    H, I, E, K, T = 7168, 256, 4, 2, 3
    g = torch.Generator(device=DEV).manual_seed(21)
    w13, s13 = synth.fp8_projection(E, 2 * I, H, g, DEV)
    w2, s2 = synth.fp8_projection(E, H, I, g, DEV)
    big = LayerWeights(lib.LAYOUT_W13_FP8_B128, H, I, E, Projection.stacked(w13, s13), Projection.stacked(w2, s2))
    eng = Engine(0, max_tokens=8, hidden=H, inter=I, experts=E, topk=K)
    x = synth.activations(T, H, g, DEV)
    idx = torch.tensor([[0, 1], [2, 3], [1, 2]], dtype=torch.int32, device=DEV)
    want = eng.expert_pairs(big, x, idx)
    eng.sync()
    small = _layer()
    small_eng = Engine(0, max_tokens=64, hidden=512, inter=256, experts=16, topk=4)
    xs = synth.activations(4, 512, g, DEV)
    out = torch.empty((4, 512), dtype=torch.bfloat16, device=DEV)
    rc, msg = _noalloc(small_eng, small, xs, 4, out)
    assert rc == lib.WM_OK, msg
    got = eng.expert_pairs(big, x, idx)
    eng.sync()
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))
    small_eng.ctx.close()
    eng.ctx.close()
