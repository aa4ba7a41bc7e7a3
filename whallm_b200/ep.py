"""Expert parallelism over the GPUs of one box (torch.distributed, NCCL).

Rank r of W owns the routed experts [r * E/W, (r + 1) * E/W); the router and
the shared expert are replicated and every rank keeps its own tokens.  One
layer forward (routing, sort, experts and combine split across GPUs):

  1. route the local tokens with the full router -> (w, idx) [T, K];
  2. wm_ep_plan orders the (t, k) pairs by owning rank (stable, so k order
     is kept per token), gathers their activation rows and owner-local
     expert ids; the per-rank pair counts are exchanged (all-to-all of W
     int32) and read on the host for the split sizes;
  3. dispatch: all-to-all-v of the rows (bf16 [n, H]) and the expert ids;
  4. the owner applies its experts to the rows it received
     (wm_expert_pairs: sort, expert kernels, unpermute);
  5. combine: the reverse all-to-all-v brings each pair's expert row back to
     the token's rank in send order, and wm_combine forms
     sum_k w[t, k] * y[t, k] + g_t * shared(x[t]) reading pair (t, k) at its
     send slot -- the same arithmetic as the single-GPU layer.  The shared
     expert of the local tokens runs on a side stream (its own handle) while
     the pairs are exchanged.

Expert rows are independent of which other rows share their GPU, so a
layer split over W GPUs returns what one GPU computes for the same tokens
whenever both take the same expert kernels (the exchanges only move rows).
The reference runs its experts on one device (model.py:181-182 refuses
more); this module is the B200-native expert-parallel layer, not a port.

With `peer_memory=True` (fixed capacity, one GPU per rank, at most 8) the
three exchanges of steps 2-5 run without the collective library: every rank
stores its pairs' rows and ids (and how many it sent) straight into the
owners' exchange buffers over NVLink; each owner plans over the real rows
only, runs its experts (decode kernels or grouped GEMM) and stores every
result row from its sorted rows straight back into the sender's buffer; and
bounded device waits on per-rank flags replace the all-to-alls
(include/whallm_moe.h, wm_ep_*).  Only real pairs cross NVLink.

The engine is anything with route / ep_plan / expert_pairs / combine of
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
    """One MoE layer whose routed experts are split evenly over a process group.

    `shared_engine`, when given, computes the shared expert on a side stream
    while the pairs are exchanged (it must be a different handle: a handle's
    workspace serves one stream at a time).

    `fixed_capacity` = M > 0 (the most tokens any rank passes in one call,
    the same on every rank): every rank sends every other rank M * K slots
    (the most pairs it can have for one rank), padding marked by expert id -1,
    so the exchanges have fixed sizes, nothing is read on the host and a step
    can be captured in a CUDA graph.  `engine` must then be a handle created
    with lib.FLAG_SKIP_NEGATIVE_ROUTES and room for W * M * K rows."""

    def __init__(self, engine, layer: LayerWeights, top_k: int, group=None, shared_engine=None,
                 fixed_capacity: int = 0, peer_memory: bool = False, owner_engine=None,
                 peer_buffer: "lib.EpBuffer | None" = None):
        if not dist.is_initialized():
            raise RuntimeError("torch.distributed is not initialised")
        self.engine, self.layer, self.K, self.group = engine, layer, top_k, group
        self.shared_engine = shared_engine
        # the handle that runs this rank's experts on the rows it receives
        # (single routes, up to world * capacity of them); the routing
        # handle's by default
        self.owner = owner_engine if owner_engine is not None else engine
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
        self.fixed = fixed_capacity
        self.stats = EPStats()
        self._side = None
        # layers that run one after another on one stream can share one exchange buffer
        self._owns_buffer = peer_memory and peer_buffer is None
        if peer_buffer is not None:
            if not peer_memory:
                raise ValueError("a peer buffer is used only with peer_memory=True")
            if (peer_buffer.world, peer_buffer.rank, peer_buffer.capacity, peer_buffer.hidden) != (
                    self.world, self.rank, self.fixed * self.K, layer.H):
                raise ValueError("the shared exchange buffer was made for another shape or group")
        self.ep_buf = peer_buffer if peer_buffer is not None else (self._open_exchange() if peer_memory else None)

    def _open_exchange(self) -> lib.EpBuffer:
        """This rank's exchange buffer, mapped into every peer (all ranks call this together)."""
        if not self.fixed:
            raise ValueError("peer-memory exchanges need a fixed capacity")
        if self.world > 8:
            raise ValueError("peer-memory exchanges support at most 8 ranks")
        ids = [None] * self.world
        dist.all_gather_object(ids, self._device_key(), group=self.group)
        if len(set(ids)) != self.world:
            raise ValueError("peer-memory exchanges need every rank on its own GPU")
        # every rank takes part in every collective below, whatever fails locally,
        # and all of them agree on the outcome
        buf, handle, error = None, b"", ""
        try:
            buf = self._new_buffer()
            handle = buf.ipc_handle()
        except lib.WMError as exc:
            error = str(exc)
        handles = [None] * self.world
        dist.all_gather_object(handles, handle, group=self.group)
        if not error:
            try:
                for r, h in enumerate(handles):
                    if r != self.rank:
                        if not h:
                            raise lib.WMError(f"rank {r} has no exchange buffer")
                        buf.open_peer(r, h)
            except lib.WMError as exc:
                error = str(exc)
        errors = [None] * self.world
        dist.all_gather_object(errors, error, group=self.group)
        if any(errors):
            if buf is not None:
                buf.close()
            raise RuntimeError("peer-memory exchange unavailable: " + "; ".join(e for e in errors if e))
        return buf

    def _device_key(self) -> str:
        """Identifies this rank's GPU across processes."""
        return str(torch.cuda.get_device_properties(self.engine.device).uuid)

    def _new_buffer(self) -> lib.EpBuffer:
        dev = self.engine.device
        return lib.EpBuffer(dev.index or 0, self.world, self.rank, self.fixed * self.K, self.layer.H)

    def close(self) -> None:
        """Release the exchange buffer once every rank has finished (collective)."""
        if self.ep_buf is not None and not self._owns_buffer:
            self.ep_buf = None
        if self.ep_buf is not None:
            if torch.cuda.is_available():
                torch.cuda.synchronize(self.engine.device)
            dist.barrier(group=self.group)
            self.ep_buf.close()
            self.ep_buf = None

    def _a2a(self, out: torch.Tensor, inp: torch.Tensor, out_splits: list[int], in_splits: list[int]) -> None:
        dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)

    def _shared_rows(self, eng, x: torch.Tensor) -> torch.Tensor:
        zero = torch.zeros((x.shape[0], 1), dtype=torch.int32, device=x.device)
        return eng.expert_pairs(self.shared, x, zero).view(x.shape[0], x.shape[1])

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        if self.layer.norm is not None:
            # the pre-MoE RMSNorm: routes, experts and the shared expert all read
            # the normalised rows, which the router writes
            xn = torch.empty_like(x)
            w, idx = self.engine.route(self.layer, x, self.K, x_norm=xn)
            x = xn
        else:
            w, idx = self.engine.route(self.layer, x, self.K)

        # the shared expert of the local tokens, beside the exchange
        shared_rows = None
        side = None
        if self.shared is not None and self.shared_engine is not None and x.is_cuda:
            if self._side is None:
                self._side = torch.cuda.Stream(device=x.device)
            side = self._side
            side.wait_stream(torch.cuda.current_stream(x.device))
            with torch.cuda.stream(side):
                shared_rows = self._shared_rows(self.shared_engine, x)

        if self.ep_buf is not None:
            back, pair_pos = self._exchange_peer(x, idx)
        elif self.fixed:
            back, pair_pos = self._exchange_fixed(x, idx)
        else:
            back, pair_pos = self._exchange_exact(x, idx)

        gate, gate_w = lib.SHARED_NONE, None
        if self.shared is not None:
            if side is not None:
                main = torch.cuda.current_stream(x.device)
                main.wait_stream(side)
                shared_rows.record_stream(main)
            else:
                shared_rows = self._shared_rows(self.engine, x)
            gate, gate_w = self.layer.shared.gate, self.layer.shared.gate_weight
        if isinstance(back, int):  # rows in the exchange buffer
            return self.engine.combine_at(back, w, shared_rows, gate, x, gate_w, pair_pos)
        return self.engine.combine(back, w, shared_rows, gate, x, gate_w, pair_pos=pair_pos)

    def _exchange_peer(self, x: torch.Tensor, idx: torch.Tensor):
        """Exchanges through the ranks' buffers over NVLink (no collective)."""
        T, H = x.shape
        if T > self.fixed:
            raise ValueError(f"{T} tokens exceed the fixed capacity of {self.fixed} per rank")
        W, El, C = self.world, self.E_local, self.fixed * self.K
        ctx, buf, stream = self.engine.ctx, self.ep_buf, torch.cuda.current_stream(x.device).cuda_stream
        idx = idx.to(torch.int32).contiguous()
        pair_pos = torch.empty((T, self.K), dtype=torch.int32, device=x.device)
        ctx.ep_dispatch(buf, T, self.K, El, idx.data_ptr(), x.data_ptr(), pair_pos.data_ptr(), stream)
        ctx.ep_wait(buf, 0, stream)
        # this rank's experts on the real rows it received; the results go
        # straight back into the senders' buffers
        self.owner.ep_experts(self.local, buf, C)
        ctx.ep_wait(buf, 1, stream)
        self.stats = EPStats(sent=-1, received=-1)
        return buf.buffer(2), pair_pos  # the result rows, in this rank's buffer

    def _exchange_fixed(self, x: torch.Tensor, idx: torch.Tensor):
        """Fixed-size exchanges: W * T * K slots each way, padding skipped."""
        T, H = x.shape
        if T > self.fixed:
            raise ValueError(f"{T} tokens exceed the fixed capacity of {self.fixed} per rank")
        W, El, C = self.world, self.E_local, self.fixed * self.K
        _, pair_pos, send_eid, send_x = self.engine.ep_plan(idx, x, El, W, capacity=C)
        recv_x = torch.empty_like(send_x)
        recv_e = torch.empty_like(send_eid)
        dist.all_to_all_single(recv_x, send_x, group=self.group)
        dist.all_to_all_single(recv_e, send_eid, group=self.group)
        y = self.owner.expert_pairs(self.local, recv_x, recv_e.view(W * C, 1)).view(W * C, H)
        back = torch.empty_like(y)
        dist.all_to_all_single(back, y, group=self.group)
        self.stats = EPStats(sent=-1, received=-1)
        return back, pair_pos

    def _exchange_exact(self, x: torch.Tensor, idx: torch.Tensor):
        """Exchanges sized by the pair counts (read on the host)."""
        T, H = x.shape
        W, El = self.world, self.E_local
        # pairs in owner order, then the counts each rank sends and receives
        send_counts, pair_pos, send_eid, send_x = self.engine.ep_plan(idx, x, El, W)
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        counts = torch.stack([send_counts, recv_counts]).cpu()  # the one host sync: split sizes
        send_splits, recv_splits = counts[0].tolist(), counts[1].tolist()
        n_send, n_recv = sum(send_splits), sum(recv_splits)

        # dispatch: activation rows and owner-local expert ids
        recv_x = torch.empty((n_recv, H), dtype=x.dtype, device=x.device)
        recv_e = torch.empty((n_recv,), dtype=torch.int32, device=x.device)
        self._a2a(recv_x, send_x, recv_splits, send_splits)
        self._a2a(recv_e, send_eid, recv_splits, send_splits)

        # this rank's experts on the rows it received
        if n_recv:
            y = self.owner.expert_pairs(self.local, recv_x, recv_e.view(n_recv, 1)).view(n_recv, H)
        else:
            y = torch.empty((0, H), dtype=x.dtype, device=x.device)

        # rows back in send order; pair (t, k) sits at pair_pos[t, k]
        back = torch.empty((n_send, H), dtype=x.dtype, device=x.device)
        self._a2a(back, y, send_splits, recv_splits)
        self.stats = EPStats(sent=n_send, received=n_recv)
        return back, pair_pos
