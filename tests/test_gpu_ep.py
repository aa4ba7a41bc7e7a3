"""Expert parallelism on GPUs (NCCL): the layer split over W ranks returns what
one GPU computes for the same tokens, and both match the CPU oracle."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from oracle import adapter
from whallm_b200 import lib, synth
from whallm_b200.moe import Engine

pytestmark = pytest.mark.gpu
H, I, E, K, B = 2048, 512, 512, 10, 64
TOL = 1e-2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _engine(dev: int, world: int) -> Engine:
    cap = world * B * K
    return Engine(dev, max_tokens=cap, hidden=H, inter=I, experts=E, topk=K, gemv_max_tokens=cap,
                  flags=lib.FLAG_SKIP_NEGATIVE_ROUTES)


def _shared_engine(dev: int) -> Engine:
    return Engine(dev, max_tokens=B, hidden=H, inter=I, experts=1, topk=1, gemv_max_tokens=B)


MODES = {"exact": (0, False), "fixed": (B, False), "peer": (B, True)}


@pytest.mark.parametrize("mode", list(MODES))
def test_ep_one_rank_equals_forward(mode):
    fixed, peer = MODES[mode]
    from whallm_b200.ep import ExpertParallelMoE
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{_free_port()}", rank=0, world_size=1,
                            device_id=torch.device("cuda", 0))
    try:
        wl = synth.config(1, device="cuda", batch=B)
        eng = _engine(0, 1)
        ep = ExpertParallelMoE(eng, wl.layer, K, shared_engine=_shared_engine(0), fixed_capacity=fixed,
                               peer_memory=peer)
        got = ep(wl.x)
        got2 = ep(wl.x)  # a second step: the exchange flags move on to the next step number
        want, (w, idx) = eng.forward(wl.layer, wl.x, K, return_routes=True)
        eng.sync()
        if not fixed:
            assert ep.stats.sent == B * K and ep.stats.received == B * K
        assert torch.equal(got, want), "expert-parallel layer (one rank) differs from the single-GPU layer"
        assert torch.equal(got2, want)
        ep.close()
        tokens = np.arange(8, dtype=np.int32)
        layer_np = adapter.from_layer(wl.layer)
        ref = layer_np.forward(adapter.bits(wl.x), idx.cpu().numpy(), w.cpu().numpy(), tokens=tokens)
        err = oracle.max_rel_error(oracle.bf16_to_f32(adapter.bits(got)[tokens]), oracle.bf16_to_f32(ref[tokens]))
        assert err <= TOL
    finally:
        dist.destroy_process_group()


def _worker(rank: int, world: int, port: int, mode: str, q) -> None:
    fixed, peer = MODES[mode]
    from whallm_b200.ep import ExpertParallelMoE
    torch.cuda.set_device(rank)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    from datetime import timedelta
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60), device_id=torch.device("cuda", rank))
    try:
        dev = torch.device("cuda", rank)
        wl = synth.config(1, device=dev, batch=B)
        x = synth.activations(B, H, torch.Generator(device=dev).manual_seed(77 + rank), dev)
        eng = _engine(rank, world)
        ep = ExpertParallelMoE(eng, wl.layer, K, shared_engine=_shared_engine(rank), fixed_capacity=fixed,
                               peer_memory=peer)
        got = ep(x)
        got2 = ep(x)
        want = eng.forward(wl.layer, x, K)
        eng.sync()
        ep.close()
        ok = bool(torch.equal(got, want)) and bool(torch.equal(got2, want))
        q.put((rank, ok, float((got.float() - want.float()).abs().max())))
    finally:
        dist.destroy_process_group()


# every world size the box can hold (2, 4, 8); a 1-GPU box runs the one-rank tests only
WORLDS = [w for w in (2, 4, 8) if w <= torch.cuda.device_count()] or [2]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("world", WORLDS)
@pytest.mark.parametrize("mode", list(MODES))
def test_ep_ranks_equal_single_gpu(mode, world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, equal, diff in res:
        assert equal, f"rank {rank}: expert-parallel output differs from one GPU (max abs diff {diff})"


def _gemm_layer(layout, E, H, I, seed):
    """A small layer of the expert-parallel long-call configs (FP8 128x128 or DS MXFP4) with a shared expert."""
    from whallm_b200.layout import Projection
    from whallm_b200.moe import LayerWeights, RouterWeights, SharedExpert
    g = torch.Generator(device="cuda").manual_seed(seed)
    proj = synth.projection_for(layout)
    w13, s13 = proj(E, 2 * I, H, g, "cuda")
    w2, s2 = proj(E, H, I, g, "cuda")
    a, b = proj(1, 2 * I, H, g, "cuda")
    c, d = proj(1, H, I, g, "cuda")
    wr = (torch.randn((E, H), generator=g, device="cuda") / H ** 0.5).to(torch.bfloat16)
    return LayerWeights(layout, H, I, E, Projection.stacked(w13, s13), Projection.stacked(w2, s2),
                        shared=SharedExpert(Projection.stacked(a, b), Projection.stacked(c, d), lib.SHARED_ONE),
                        router=RouterWeights(wr, lib.ROUTER_SIGMOID))


@pytest.mark.parametrize("layout", [lib.LAYOUT_W13_FP8_B128, lib.LAYOUT_DS_W13_MXFP4])
def test_ep_grouped_gemm_owner_equals_forward(layout):
    """The owner half on the grouped GEMM (wm_ep_experts: plan over the real
    rows of each block, experts, result rows straight back from the sorted
    rows) over peer memory, one rank: bit-identical to the one-GPU layer on
    the grouped GEMM, two steps in a row, and within tolerance of the oracle."""
    from whallm_b200.ep import ExpertParallelMoE
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{_free_port()}", rank=0, world_size=1,
                            device_id=torch.device("cuda", 0))
    try:
        E_, H_, I_, K_, T_ = 16, 1024, 512, 4, 300
        layer = _gemm_layer(layout, E_, H_, I_, seed=90 + layout)
        x = synth.activations(T_, H_, torch.Generator(device="cuda").manual_seed(91), "cuda")
        eng = Engine(0, max_tokens=T_, hidden=H_, inter=I_, experts=E_, topk=K_, gemv_max_tokens=-1)
        owner = Engine(0, max_tokens=T_ * K_, hidden=H_, inter=I_, experts=E_, topk=1, gemv_max_tokens=-1)
        shared = Engine(0, max_tokens=T_, hidden=H_, inter=I_, experts=1, topk=1, gemv_max_tokens=-1)
        ep = ExpertParallelMoE(eng, layer, K_, shared_engine=shared, fixed_capacity=T_, peer_memory=True,
                               owner_engine=owner)
        got, got2 = ep(x), ep(x)
        want, (w, idx) = eng.forward(layer, x, K_, return_routes=True)
        eng.sync()
        owner.sync()
        assert owner.ctx.counters().gemm_calls == 2
        assert torch.equal(got.view(torch.int16), want.view(torch.int16))
        assert torch.equal(got2.view(torch.int16), want.view(torch.int16))
        ep.close()
        tokens = np.arange(0, T_, 37, dtype=np.int32)
        ref = adapter.from_layer(layer).forward(adapter.bits(x), idx.cpu().numpy(), w.cpu().numpy(), tokens=tokens)
        err = oracle.max_rel_error(oracle.bf16_to_f32(adapter.bits(got)[tokens]), oracle.bf16_to_f32(ref[tokens]))
        assert err <= TOL
        for e_ in (eng, owner, shared):
            e_.ctx.close()
    finally:
        dist.destroy_process_group()


def test_ep_wait_times_out_without_a_peer_and_handle_stays_usable():
    """The bounded flag wait gives up when no peer ever signals: a dispatch
    bumps the step number, then a wait for returned rows that no peer sends
    (no wm_ep_return) runs out after its 2 s limit, records the timeout in
    the device status (wm_sync reports it) and returns -- the GPU and the
    handle stay usable, and a normal layer call then succeeds."""
    wl = synth.config(1, device="cuda", batch=8)
    eng = _engine(0, 1)
    buf = lib.EpBuffer(0, 1, 0, 8 * K, H)
    try:
        x = wl.x
        _, idx = eng.route(wl.layer, x, K)
        pair_pos = torch.empty((8, K), dtype=torch.int32, device="cuda")
        stream = torch.cuda.current_stream().cuda_stream
        eng.ctx.ep_dispatch(buf, 8, K, E, idx.data_ptr(), x.data_ptr(), pair_pos.data_ptr(), stream)
        eng.ctx.ep_wait(buf, 0, stream)  # this rank's own dispatch flag: arrives
        eng.sync()
        eng.ctx.ep_wait(buf, 1, stream)  # nothing returns the rows: runs out
        with pytest.raises(lib.WMError, match="return wait timed out"):
            eng.sync()
        eng.sync()  # the record was cleared when it was reported
        out = eng.forward(wl.layer, x, K)
        eng.sync()
        assert torch.isfinite(out.float()).all()
    finally:
        buf.close()
        eng.ctx.close()
