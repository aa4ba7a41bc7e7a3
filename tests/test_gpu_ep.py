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


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("mode", list(MODES))
def test_ep_two_ranks_equal_single_gpu(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, equal, diff in res:
        assert equal, f"rank {rank}: expert-parallel output differs from one GPU (max abs diff {diff})"
