"""Expert parallelism over the GPUs of one box (torch.distributed, NCCL).

Rank r of W owns the routed experts [r * E/W, (r + 1) * E/W); the router and
the shared expert are replicated and every rank keeps its own tokens.  One
layer forward (the survey's hot-path rows a6-a8 split across GPUs):

  1. route the local tokens with the full router -> (w, idx) [T, K];
  2. order the (t, k) pairs by owning rank (stable, so k order is kept per
     token) and exchange the per-rank pair counts (all-to-all of W int32);
  3. dispatch: all-to-all-v of the pairs' activation rows (bf16 [n, H]) and
     their expert ids local to the owner (int32 [n]);
  4. the owner applies its experts to the rows it received
     (wm_expert_pairs: sort, expert kernels, unpermute);
  5. combine: the reverse all-to-all-v brings each pair's expert row back to
     the token's rank, which scatters it to (t, k) order and forms
     sum_k w[t, k] * y[t, k] + g_t * shared(x[t]) with wm_combine -- the same
     arithmetic as the single-GPU layer.

Expert rows are independent of which other rows share their GPU, so a
layer split over W GPUs returns what one GPU computes for the same tokens
whenever both take the same expert kernels (the exchanges only move rows).
The reference runs its experts on one device; this module is the
B200-native counterpart of the survey's expert-parallel plan, not a port.

The engine is anything with route / expert_pairs / combine of
whallm_b200.moe.Engine's signatures, so the exchange logic can be tested with
CPU stand-ins on gloo.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

from . import lib
from .moe import LayerWeights


@dataclass
class EPStats:
    """Pairs this rank sent and received in its last forward."""
    sent: int = 0
    received: int = 0


class ExpertParallelMoE:
    """One MoE layer whose routed experts are split evenly over a process group."""

    def __init__(self, engine, layer: LayerWeights, top_k: int, group=None):
        if not dist.is_initialized():
            raise RuntimeError("torch.distributed is not initialised")
        self.engine, self.layer, self.K, self.group = engine, layer, top_k, group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if layer.E % self.world:
            raise ValueError(f"{layer.E} experts do not split evenly over {self.world} ranks")
        if layer.router is None:
            raise ValueError("expert parallelism routes on every rank: the layer needs its router weights")
        self.E_local = layer.E // self.world
        e0 = self.rank * self.E_local
        self.local = layer.experts(e0, e0 + self.E_local)
        self.shared = layer.shared_only() if layer.shared is not None else None
        self.stats = EPStats()

    def _a2a(self, out: torch.Tensor, inp: torch.Tensor, out_splits: list[int], in_splits: list[int]) -> None:
        dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        T, H = x.shape
        K, W, El = self.K, self.world, self.E_local
        w, idx = self.engine.route(self.layer, x, K)
        flat = idx.reshape(-1).to(torch.int64)
        owner = torch.div(flat, El, rounding_mode="floor")
        order = torch.argsort(owner, stable=True)
        send_counts = torch.bincount(owner, minlength=W).to(torch.int64)
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        counts = torch.stack([send_counts, recv_counts]).cpu()  # the one host sync: split sizes
        send_splits, recv_splits = counts[0].tolist(), counts[1].tolist()
        n_send, n_recv = sum(send_splits), sum(recv_splits)

        # dispatch: activation rows and owner-local expert ids, grouped by owner
        send_x = x.index_select(0, torch.div(order, K, rounding_mode="floor"))
        send_e = (flat.index_select(0, order) - owner.index_select(0, order) * El).to(torch.int32)
        recv_x = torch.empty((n_recv, H), dtype=x.dtype, device=x.device)
        recv_e = torch.empty((n_recv,), dtype=torch.int32, device=x.device)
        self._a2a(recv_x, send_x, recv_splits, send_splits)
        self._a2a(recv_e, send_e, recv_splits, send_splits)

        # this rank's experts on the rows it received
        if n_recv:
            y = self.engine.expert_pairs(self.local, recv_x, recv_e.view(n_recv, 1)).view(n_recv, H)
        else:
            y = torch.empty((0, H), dtype=x.dtype, device=x.device)

        # combine: rows back to the tokens' ranks, then (t, k) order
        back = torch.empty((n_send, H), dtype=x.dtype, device=x.device)
        self._a2a(back, y, send_splits, recv_splits)
        pairs = torch.empty((T * K, H), dtype=x.dtype, device=x.device)
        pairs.index_copy_(0, order, back)

        shared_rows, gate, gate_w = None, lib.SHARED_NONE, None
        if self.shared is not None:
            zero = torch.zeros((T, 1), dtype=torch.int32, device=x.device)
            shared_rows = self.engine.expert_pairs(self.shared, x, zero).view(T, H)
            gate, gate_w = self.layer.shared.gate, self.layer.shared.gate_weight
        self.stats = EPStats(sent=n_send, received=n_recv)
        return self.engine.combine(pairs.view(T, K, H), w, shared_rows, gate, x, gate_w)
