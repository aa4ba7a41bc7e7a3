"""Expert-parallel exchange logic (whallm_b200.ep) on CPU: gloo ranks, a CPU
stand-in engine with dense experts.

Each rank routes its own tokens, dispatches the pairs to the experts' owners
with all-to-all, gets the expert rows back and combines them; the result must
equal, bit for bit, a single process applying every expert to the same
tokens (the exchanges only move rows).  Covers uneven pair counts, a rank
that receives no pairs, and the shared expert."""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from whallm_b200 import lib
from whallm_b200.layout import Projection
from whallm_b200.moe import LayerWeights, RouterWeights, SharedExpert

H, I, E, K = 32, 16, 8, 3


def _layer(seed: int, shared: bool) -> LayerWeights:
    g = torch.Generator().manual_seed(seed)
    w13 = torch.randn((E, 2 * I, H), generator=g) / H ** 0.5
    w2 = torch.randn((E, H, I), generator=g) / I ** 0.5
    dummy = torch.zeros((E, 1, 1))
    sh = None
    if shared:
        a = torch.randn((1, 2 * I, H), generator=g) / H ** 0.5
        b = torch.randn((1, H, I), generator=g) / I ** 0.5
        gate = (torch.randn((H,), generator=g) / H ** 0.5).to(torch.bfloat16)
        sh = SharedExpert(Projection.stacked(a, torch.zeros((1, 1, 1))), Projection.stacked(b, torch.zeros((1, 1, 1))),
                          lib.SHARED_SIGMOID_GATE, gate)
    wr = (torch.randn((E, H), generator=g) / H ** 0.5).to(torch.bfloat16)
    return LayerWeights(lib.LAYOUT_QWEN_GATE_UP_MXFP4, H, I, E, Projection.stacked(w13, dummy),
                        Projection.stacked(w2, dummy), shared=sh, router=RouterWeights(wr, lib.ROUTER_SOFTMAX))


class CpuEngine:
    """Deterministic per-row stand-in for whallm_b200.moe.Engine."""

    def route(self, layer, x, k):
        logits = x.double() @ layer.router.weight.double().t()
        top, idx = torch.topk(torch.softmax(logits, -1), k, dim=-1)
        return (top / top.sum(-1, keepdim=True)).float(), idx.to(torch.int32)

    def expert_pairs(self, layer, x, indices):
        T = x.shape[0]
        idx = indices.reshape(T, -1)
        out = torch.empty((T, idx.shape[1], layer.H), dtype=torch.bfloat16)
        for t in range(T):
            for k in range(idx.shape[1]):
                e = int(idx[t, k])
                if e < 0:  # padding slot of a fixed-capacity exchange
                    out[t, k] = 0
                    continue
                gu = layer.w13.weight[e].double() @ x[t].double()
                act = torch.nn.functional.silu(gu[:layer.I]) * gu[layer.I:]
                out[t, k] = (layer.w2.weight[e].double() @ act).to(torch.bfloat16)
        return out

    def ep_plan(self, idx, x, per_rank, world, capacity=0):
        T, k = idx.shape
        owner = (idx.reshape(-1).long() // per_rank)
        order = torch.argsort(owner, stable=True)
        pair_pos = torch.empty_like(order)
        pair_pos[order] = torch.arange(order.numel())
        counts = torch.bincount(owner, minlength=world).to(torch.int32)
        send_eid = (idx.reshape(-1).long()[order] % per_rank).to(torch.int32)
        send_x = x[order // k]
        if capacity:
            starts = torch.cumsum(counts, 0) - counts
            slot = owner[order] * capacity + (torch.arange(order.numel()) - starts[owner[order]])
            eid = torch.full((world * capacity,), -1, dtype=torch.int32)
            rows = torch.zeros((world * capacity, x.shape[1]), dtype=x.dtype)
            eid[slot] = send_eid
            rows[slot] = send_x
            pair_pos[order] = slot
            send_eid, send_x = eid, rows
        return counts, pair_pos.view(T, k).to(torch.int32), send_eid, send_x

    def combine(self, pairs, w, shared_rows=None, shared_gate=lib.SHARED_NONE, x=None, gate_weight=None,
                pair_pos=None):
        T, k = w.shape
        if pair_pos is not None:
            pairs = pairs[pair_pos.reshape(-1).long()].view(T, k, -1)
        acc = torch.zeros((T, pairs.shape[2]), dtype=torch.float32)
        for j in range(k):
            acc = acc + w[:, j:j + 1] * pairs[:, j].float()
        if shared_gate != lib.SHARED_NONE:
            g = torch.sigmoid(x.float() @ gate_weight.float()) if shared_gate == lib.SHARED_SIGMOID_GATE \
                else torch.ones((T,))
            acc = acc + g[:, None] * shared_rows.float()
        return acc.to(torch.bfloat16)

    def forward(self, layer, x, k):
        w, idx = self.route(layer, x, k)
        pairs = self.expert_pairs(layer, x, idx)
        sr, gate, gw = None, lib.SHARED_NONE, None
        if layer.shared is not None:
            sr = self.expert_pairs(layer.shared_only(), x, torch.zeros((x.shape[0], 1), dtype=torch.int32))[:, 0]
            gate, gw = layer.shared.gate, layer.shared.gate_weight
        return self.combine(pairs, w, sr, gate, x, gw)


def _tokens(rank: int, n: int) -> torch.Tensor:
    return torch.randn((n, H), generator=torch.Generator().manual_seed(100 + rank)).to(torch.bfloat16)


def _worker(rank: int, world: int, port: int, shared: bool, skew: bool, fixed: bool, q) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from whallm_b200.ep import ExpertParallelMoE
        layer = _layer(7, shared)
        if skew:  # every token prefers experts 0..K-1, all owned by rank 0: rank 1 receives nothing
            w = layer.router.weight.clone()
            w[:K] = 0
            w[:K, 0] = 50
            layer.router = RouterWeights(w, lib.ROUTER_SOFTMAX)
        eng = CpuEngine()
        x = _tokens(rank, 5 + 4 * rank)  # uneven token counts per rank
        if skew:
            x[:, 0] = 1.0
        ep = ExpertParallelMoE(eng, layer, K, fixed_capacity=16 if fixed else 0)
        got = ep(x)
        want = eng.forward(layer, x, K)
        q.put((rank, bool(torch.equal(got, want)), ep.stats.sent, ep.stats.received))
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("shared,skew,fixed", [(True, False, False), (False, False, False), (True, True, False),
                                               (True, False, True), (True, True, True)])
def test_ep_matches_single_process(shared, skew, fixed):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    world = 2
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, shared, skew, fixed, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    results.sort()
    for rank, equal, sent, received in results:
        assert equal, f"rank {rank}: expert-parallel output differs from the single-process layer"
        if not fixed:
            assert sent == (5 + 4 * rank) * K
    if skew and not fixed:
        assert results[1][3] == 0  # rank 1 owns no chosen expert



class _FakeBuffer:
    """Stands in for lib.EpBuffer; fails where told to."""

    def __init__(self, fail_open: bool):
        self.fail_open, self.opened, self.closed = fail_open, [], False

    def ipc_handle(self) -> bytes:
        return b"h" * 64

    def open_peer(self, peer: int, handle: bytes) -> None:
        if self.fail_open:
            raise lib.WMError(f"cannot map rank {peer}")
        self.opened.append(peer)

    def close(self) -> None:
        self.closed = True


def _setup_worker(rank: int, world: int, port: int, case: str, q) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from whallm_b200.ep import ExpertParallelMoE

        made = []

        class Probe(ExpertParallelMoE):
            def _device_key(self) -> str:
                return "gpu-0" if case == "same_gpu" else f"gpu-{rank}"

            def _new_buffer(self):
                if case == "create_fails" and rank == 1:
                    raise lib.WMError("no device memory")
                made.append(_FakeBuffer(fail_open=case == "open_fails" and rank == 0))
                return made[-1]

        try:
            ep = Probe(CpuEngine(), _layer(7, False), K, fixed_capacity=4, peer_memory=True)
            q.put((rank, "ok", made[0].opened, False))
            ep.ep_buf = None
        except (RuntimeError, ValueError) as exc:
            q.put((rank, type(exc).__name__ + ": " + str(exc), [], bool(made) and made[0].closed))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("case", ["ok", "create_fails", "open_fails", "same_gpu"])
def test_peer_exchange_setup_agrees_on_every_rank(case):
    """A buffer that cannot be created or mapped on any rank makes every rank
    give up the peer-memory exchange together (so all of them fall back to the
    collective path instead of waiting on each other); ranks sharing a GPU are
    refused."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_setup_worker, args=(r, 2, port, case, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    outcomes = [r[1] for r in res]
    if case == "ok":
        assert outcomes == ["ok", "ok"] and res[0][2] == [1] and res[1][2] == [0]
    elif case == "same_gpu":
        assert all(o.startswith("ValueError") for o in outcomes)
    else:
        assert all(o.startswith("RuntimeError: peer-memory exchange unavailable") for o in outcomes), outcomes
        assert all(("no device memory" if case == "create_fails" else "cannot map") in o for o in outcomes)
        for rank, _, _, closed in res:  # a buffer that was made is released
            if case == "open_fails" or rank == 0:
                assert closed
