"""PyTorch front end of the MoE expert-FFN path.

``Engine`` owns one library handle per device and enqueues every call on the
current PyTorch CUDA stream.  The classes below it keep the call shapes of the
reference's Python layer, so a caller switches by swapping the module:

  StreamingExperts.__call__(value [1, T, H], indices [1, T, K]) -> [1, T, K, H]
      runtime/deepseek_v4_ssd/qwen4_exp.py:797-904
  SparseMoE.route(value) / __call__(value, routes=None) -> [1, T, H]
      qwen4_exp.py:998-1051
  StreamingSwitchGLU.__call__(x, indices) -> [..., K, H]      model.py:318-501
  streaming_moe(x) (gate -> shared -> routed -> reduce)        model.py:526-546
  MoE (DeepSeek V4.1: clamped SwiGLU, sqrt-softplus gate)      deepseek_v41/moe.py:96-112

Weights are the blob bytes as [E, ...] tensor views (layout.QwenBatchedExperts
and friends), exactly as ExpertCache.current_batched returns them.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch

from . import lib
from .layout import FP8BatchedExperts, Projection, QwenBatchedExperts, projections

__all__ = [
    "Engine", "LayerWeights", "PreNorm", "RouterWeights", "SharedExpert",
    "StreamingExperts", "SparseMoE", "StreamingSwitchGLU", "MoE",
]


@dataclass
class SharedExpert:
    """The shared expert: one blob in the layer's layout, and its gate kind."""
    w13: Projection
    w2: Projection
    gate: int = lib.SHARED_ONE            # SHARED_SIGMOID_GATE (Qwen) or SHARED_ONE (DeepSeek)
    gate_weight: torch.Tensor | None = None  # bf16 [H] for the sigmoid gate


@dataclass
class RouterWeights:
    weight: torch.Tensor                   # bf16 [E, H]
    kind: int = lib.ROUTER_SOFTMAX
    bias: torch.Tensor | None = None       # fp32 [E]
    n_groups: int = 1
    topk_groups: int = 1
    route_scale: float = 1.0


@dataclass
class PreNorm:
    """The RMSNorm in front of the MoE block (post_attention_layernorm):
    xn = bf16((x * rsqrt(mean(x^2) + eps)) * weight), engine.mm:1846 with
    kernels.metal:443-465 (rms_norm_tg), GroupRMSNorm in qwen4_exp.py:93-117."""
    weight: torch.Tensor                   # bf16 [H]
    eps: float = 1e-6


@dataclass
class LayerWeights:
    """Everything of one MoE layer the expert kernels read."""
    layout: int
    H: int
    I: int
    E: int
    w13: Projection
    w2: Projection
    shared: SharedExpert | None = None
    router: RouterWeights | None = None
    swiglu_limit: float = 0.0
    norm: PreNorm | None = None            # applied to x first when set
    keep: list = field(default_factory=list)  # tensors the views point into

    @staticmethod
    def from_batched(batched, H: int, I: int, **kw) -> "LayerWeights":
        layout, w13, w2 = projections(batched)
        return LayerWeights(layout, H, I, w13.weight.shape[0], w13, w2, keep=[batched], **kw)

    def experts(self, e0: int, e1: int) -> "LayerWeights":
        """Routed experts [e0, e1) only (views, no copy): an expert-parallel shard."""
        if not 0 <= e0 < e1 <= self.E:
            raise ValueError(f"expert range [{e0}, {e1}) outside [0, {self.E})")
        def cut(p: Projection) -> Projection:
            return Projection(p.weight[e0:e1], p.weight_stride, p.scale[e0:e1], p.scale_stride)
        return LayerWeights(self.layout, self.H, self.I, e1 - e0, cut(self.w13), cut(self.w2),
                            swiglu_limit=self.swiglu_limit, keep=self.keep)

    def shared_only(self) -> "LayerWeights":
        """The shared expert as a one-expert layer."""
        if self.shared is None:
            raise ValueError("the layer has no shared expert")
        return LayerWeights(self.layout, self.H, self.I, 1, self.shared.w13, self.shared.w2,
                            swiglu_limit=self.swiglu_limit, keep=self.keep)


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _check_bf16(name: str, t: torch.Tensor, shape: tuple[int, ...] | None = None) -> None:
    if t.dtype != torch.bfloat16 or not t.is_cuda or not t.is_contiguous():
        raise ValueError(f"{name} must be a contiguous bf16 CUDA tensor")
    if shape is not None and tuple(t.shape) != shape:
        raise ValueError(f"{name} has shape {tuple(t.shape)}, expected {shape}")


def _check_shape_bf16(name: str, t: torch.Tensor, shape: tuple[int, ...]) -> None:
    """bf16 of the given shape, on the device or on the host (pinned for overlap)."""
    if t.dtype != torch.bfloat16 or tuple(t.shape) != shape:
        raise ValueError(f"{name} must be bf16 {shape}, got {t.dtype} {tuple(t.shape)}")


class Engine:
    """A library handle sized for the largest call it will see."""

    def __init__(self, device: int | torch.device = 0, *, max_tokens: int, hidden: int, inter: int, experts: int,
                 topk: int, gemv_max_tokens: int = 0, flags: int = 0):
        dev = torch.device("cuda", device) if isinstance(device, int) else torch.device(device)
        if dev.type != "cuda":
            raise ValueError("the expert kernels run on CUDA devices only")
        self.device = dev
        with torch.cuda.device(dev):
            self.ctx = lib.Context(dev.index or 0, max_tokens=max_tokens, max_hidden=hidden, max_inter=inter,
                                   max_experts=experts, max_topk=topk, gemv_max_tokens=gemv_max_tokens,
                                   flags=flags)

    # ---------------------------------------------------------------- argument block
    def _args(self, layer: LayerWeights, x: torch.Tensor, K: int) -> lib.MoeArgs:
        T = x.shape[0]
        _check_bf16("x", x, (T, layer.H))
        return self._args_at(layer, T, x.data_ptr(), K)

    def _args_at(self, layer: LayerWeights, T: int, x_ptr: int, K: int) -> lib.MoeArgs:
        a = lib.MoeArgs()
        a.T, a.H, a.I, a.E, a.K = T, layer.H, layer.I, layer.E, K
        a.layout = layer.layout
        a.w13 = layer.w13.matrix()
        a.w2 = layer.w2.matrix()
        a.x = x_ptr
        a.swiglu_limit = layer.swiglu_limit
        a.route_scale = 1.0
        if layer.norm is not None:
            _check_bf16("norm weight", layer.norm.weight, (layer.H,))
            a.norm_weight = layer.norm.weight.data_ptr()
            a.norm_eps = layer.norm.eps
        return a

    @staticmethod
    def _with_x_norm(a: lib.MoeArgs, layer: LayerWeights, x: torch.Tensor, x_norm: torch.Tensor | None) -> None:
        if x_norm is None:
            return
        if layer.norm is None:
            raise ValueError("x_norm is written only for layers with a pre-MoE norm")
        _check_bf16("x_norm", x_norm, tuple(x.shape))
        a.x_norm = x_norm.data_ptr()

    def _with_shared(self, a: lib.MoeArgs, layer: LayerWeights) -> None:
        if layer.shared is None:
            a.shared_gate = lib.SHARED_NONE
            return
        a.shared_w13 = layer.shared.w13.matrix()
        a.shared_w2 = layer.shared.w2.matrix()
        a.shared_gate = layer.shared.gate
        a.shared_gate_weight = _ptr(layer.shared.gate_weight)

    def _with_router(self, a: lib.MoeArgs, r: RouterWeights) -> None:
        a.router = r.kind
        a.router_weight = r.weight.data_ptr()
        a.router_bias = _ptr(r.bias)
        a.n_groups, a.topk_groups, a.route_scale = r.n_groups, r.topk_groups, r.route_scale

    # ---------------------------------------------------------------- calls
    def route(self, layer: LayerWeights, x: torch.Tensor, K: int, with_logits: bool = False,
              x_norm: torch.Tensor | None = None):
        """(weights fp32 [T, K], indices int32 [T, K][, logits fp32 [T, E]]).
        With layer.norm the routes are those of the normalised rows (written
        to x_norm when given)."""
        if layer.router is None:
            raise ValueError("the layer has no router weights")
        a = self._args(layer, x, K)
        self._with_x_norm(a, layer, x, x_norm)
        self._with_router(a, layer.router)
        T = x.shape[0]
        idx = torch.empty((T, K), dtype=torch.int32, device=x.device)
        w = torch.empty((T, K), dtype=torch.float32, device=x.device)
        logits = torch.empty((T, layer.E), dtype=torch.float32, device=x.device) if with_logits else None
        self.ctx.route(a, _ptr(logits), idx.data_ptr(), w.data_ptr(), _stream())
        return (w, idx, logits) if with_logits else (w, idx)

    def expert_pairs(self, layer: LayerWeights, x: torch.Tensor, indices: torch.Tensor,
                     x_norm: torch.Tensor | None = None) -> torch.Tensor:
        """routed bf16 [T, K, H]: row (t, k) = expert indices[t, k] applied to x[t]
        (to the normalised x[t] with layer.norm)."""
        T = x.shape[0]
        idx = indices.reshape(T, -1).to(torch.int32).contiguous()
        K = idx.shape[1]
        a = self._args(layer, x, K)
        self._with_x_norm(a, layer, x, x_norm)
        a.routes_idx = idx.data_ptr()
        out = torch.empty((T, K, layer.H), dtype=torch.bfloat16, device=x.device)
        self.ctx.expert_pairs(a, out.data_ptr(), _stream())
        return out

    def forward(self, layer: LayerWeights, x: torch.Tensor, K: int, routes: tuple | None = None,
                out: torch.Tensor | None = None, return_routes: bool = False,
                x_norm: torch.Tensor | None = None):
        """Combined output bf16 [T, H].  `routes` = (weights fp32 [T, K], indices
        int32 [T, K]) skips the router.  With layer.norm every part of the block
        reads the normalised rows, which x_norm (bf16 [T, H]) receives when given."""
        T = x.shape[0]
        a = self._args(layer, x, K)
        self._with_x_norm(a, layer, x, x_norm)
        self._with_shared(a, layer)
        keep = []
        if routes is None:
            self._with_router(a, layer.router)
            if return_routes:
                ri = torch.empty((T, K), dtype=torch.int32, device=x.device)
                rw = torch.empty((T, K), dtype=torch.float32, device=x.device)
                a.out_idx, a.out_w = ri.data_ptr(), rw.data_ptr()
        else:
            rw, ri = routes
            rw = rw.reshape(T, K).to(torch.float32).contiguous()
            ri = ri.reshape(T, K).to(torch.int32).contiguous()
            keep += [rw, ri]
            a.routes_idx, a.routes_w = ri.data_ptr(), rw.data_ptr()
        if out is None:
            out = torch.empty((T, layer.H), dtype=torch.bfloat16, device=x.device)
        _check_bf16("out", out, (T, layer.H))
        a.out = out.data_ptr()
        self.ctx.moe_forward(a, _stream())
        if return_routes:
            return out, (rw, ri)
        return out

    def expert_pairs_at(self, layer: LayerWeights, T: int, x_ptr: int, idx_ptr: int, out: torch.Tensor) -> torch.Tensor:
        """expert_pairs on rows that live outside torch (an exchange buffer):
        x bf16 [T, H] at x_ptr, one route per row (int32 [T] at idx_ptr); out bf16 [T, H]."""
        _check_bf16("out", out, (T, layer.H))
        a = self._args_at(layer, T, x_ptr, 1)
        a.routes_idx = idx_ptr
        self.ctx.expert_pairs(a, out.data_ptr(), _stream())
        return out

    def ep_experts(self, layer: LayerWeights, buf: "lib.EpBuffer", expected_rows: int) -> None:
        """The owner's half of a peer-memory expert-parallel step (after the
        dispatch wait): `layer`'s experts (this rank's shard) on the rows the
        peers sent, results stored straight into the senders' buffers.
        expected_rows picks the expert kernels (decode or grouped GEMM)."""
        a = lib.MoeArgs()
        a.T, a.H, a.I, a.E, a.K = expected_rows, layer.H, layer.I, layer.E, 1
        a.layout = layer.layout
        a.w13 = layer.w13.matrix()
        a.w2 = layer.w2.matrix()
        a.swiglu_limit = layer.swiglu_limit
        a.route_scale = 1.0
        self.ctx.ep_experts(buf, a, _stream())

    def combine(self, pairs: torch.Tensor, w: torch.Tensor, shared_rows: torch.Tensor | None = None,
                shared_gate: int = lib.SHARED_NONE, x: torch.Tensor | None = None,
                gate_weight: torch.Tensor | None = None, out: torch.Tensor | None = None,
                pair_pos: torch.Tensor | None = None) -> torch.Tensor:
        """out[t] = sum_k w[t, k] * y(t, k) + g_t * shared_rows[t] (bf16 [T, H]), the same
        arithmetic as forward's combine.  y(t, k) = pairs[t, k] for pairs bf16 [T, K, H],
        or pairs[pair_pos[t, k]] for pairs bf16 [rows, H] with pair_pos int32 [T, K]."""
        T, K = w.shape
        H = pairs.shape[-1]
        if pair_pos is None:
            _check_bf16("pairs", pairs, (T, K, H))
        else:
            _check_bf16("pairs", pairs, (pairs.shape[0], H))
            pair_pos = pair_pos.reshape(T, K).to(torch.int32).contiguous()
        w = w.reshape(T, K).to(torch.float32).contiguous()
        if shared_gate != lib.SHARED_NONE:
            _check_bf16("shared_rows", shared_rows, (T, H))
        if out is None:
            out = torch.empty((T, H), dtype=torch.bfloat16, device=pairs.device)
        self.ctx.combine(T, H, K, pairs.data_ptr(), _ptr(pair_pos), w.data_ptr(), _ptr(shared_rows), shared_gate,
                         _ptr(x), _ptr(gate_weight), out.data_ptr(), _stream())
        return out

    def combine_at(self, pairs_ptr: int, w: torch.Tensor, shared_rows: torch.Tensor | None,
                   shared_gate: int, x: torch.Tensor | None, gate_weight: torch.Tensor | None,
                   pair_pos: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """combine over pair rows outside torch (bf16 [*, H] at pairs_ptr), pair (t, k) at row pair_pos[t, k]."""
        T, K = w.shape
        H = x.shape[1]
        pair_pos = pair_pos.reshape(T, K).to(torch.int32).contiguous()
        w = w.reshape(T, K).to(torch.float32).contiguous()
        if shared_gate != lib.SHARED_NONE:
            _check_bf16("shared_rows", shared_rows, (T, H))
        if out is None:
            out = torch.empty((T, H), dtype=torch.bfloat16, device=x.device)
        self.ctx.combine(T, H, K, pairs_ptr, pair_pos.data_ptr(), w.data_ptr(), _ptr(shared_rows), shared_gate,
                         _ptr(x), _ptr(gate_weight), out.data_ptr(), _stream())
        return out

    def ep_plan(self, idx: torch.Tensor, x: torch.Tensor, per_rank: int, world: int, capacity: int = 0):
        """Dispatch plan of routes idx [T, K] over `world` ranks of `per_rank`
        experts: (send_counts int32 [world], pair_pos int32 [T, K], send_eid int32
        [slots], send_x bf16 [slots, H]) -- pairs in owner order, x rows per slot;
        slots = T * K packed, or world * capacity with padding ids -1."""
        T, K = idx.shape
        H = x.shape[1]
        idx = idx.to(torch.int32).contiguous()
        _check_bf16("x", x, (T, H))
        dev = x.device
        slots = world * capacity if capacity else T * K
        counts = torch.empty((world,), dtype=torch.int32, device=dev)
        pair_pos = torch.empty((T, K), dtype=torch.int32, device=dev)
        send_eid = torch.empty((slots,), dtype=torch.int32, device=dev)
        send_x = torch.empty((slots, H), dtype=torch.bfloat16, device=dev)
        self.ctx.ep_plan(T, K, per_rank, world, capacity, idx.data_ptr(), x.data_ptr(), H, counts.data_ptr(),
                         pair_pos.data_ptr(), send_eid.data_ptr(), send_x.data_ptr(), _stream())
        return counts, pair_pos, send_eid, send_x

    def dequant(self, fmt: int, weight: torch.Tensor, scale: torch.Tensor, rows: int, cols: int,
                convention: int = lib.CONV_MLX) -> torch.Tensor:
        out = torch.empty((rows, cols), dtype=torch.bfloat16, device=weight.device)
        self.ctx.dequant(fmt, weight.data_ptr(), scale.data_ptr(), rows, cols, convention, out.data_ptr(), _stream())
        return out

    def sync(self) -> None:
        """Wait for the current stream and raise any error a kernel recorded."""
        self.ctx.sync(_stream())

    # ---------------------------------------------------------------- replayed calls
    def replay(self, layer: LayerWeights, x: torch.Tensor, K: int, out: torch.Tensor | None = None) -> torch.Tensor:
        """forward() of a repeated call shape (decode) from a CUDA graph.

        The first call for a (layer, T, K) runs the layer once and captures it
        into a graph over a static input and output block on this device; every
        later call copies x into the input block, replays the graph and copies
        the output block into out.  x and out may be device tensors or pinned
        host tensors (the copies then cross PCIe straight into and out of the
        static blocks).  Results equal forward()'s bit for bit.  The graph keeps
        the layer's weight pointers: call release_replays() after replacing a
        layer's tensors.  Calls are stream-ordered on the current stream."""
        T = x.shape[0]
        _check_shape_bf16("x", x, (T, layer.H))
        if T == 0:  # nothing to run (and nothing worth a graph)
            if out is None:
                out = torch.empty((0, layer.H), dtype=torch.bfloat16, device=self.device)
            _check_shape_bf16("out", out, (0, layer.H))
            return out
        key = (id(layer), T, K)
        entry = getattr(self, "_replays", {}).get(key)
        if entry is None:
            entry = self._capture(layer, T, K)
        graph, xs, os_, _ = entry
        xs.copy_(x, non_blocking=True)
        graph.replay()
        if out is None:
            out = torch.empty((T, layer.H), dtype=torch.bfloat16, device=self.device)
        _check_shape_bf16("out", out, (T, layer.H))
        out.copy_(os_, non_blocking=True)
        return out

    def _capture(self, layer: LayerWeights, T: int, K: int):
        if not hasattr(self, "_replays"):
            self._replays = {}
        xs = torch.zeros((T, layer.H), dtype=torch.bfloat16, device=self.device)
        os_ = torch.empty((T, layer.H), dtype=torch.bfloat16, device=self.device)
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            self.forward(layer, xs, K, out=os_)  # first launches (kernel attributes) outside the capture
        torch.cuda.current_stream(self.device).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            self.forward(layer, xs, K, out=os_)
        entry = (graph, xs, os_, layer)  # the layer stays referenced while its graph lives
        self._replays[(id(layer), T, K)] = entry
        return entry

    def release_replays(self) -> None:
        """Drop every captured call shape (and its static blocks)."""
        self._replays = {}


# -------------------------------------------------------------------- reference-shaped wrappers

class StreamingExperts:
    """qwen4_exp.StreamingExperts: routed rows of the batched layer, no combine."""

    def __init__(self, layer: int, cache, engine: Engine):
        self.layer, self.cache, self.engine = layer, cache, engine

    def __call__(self, value: torch.Tensor, indices: torch.Tensor) -> torch.Tensor:
        batched = self.cache.current_batched(self.layer)
        H = value.shape[-1]
        lw = LayerWeights.from_batched(batched, H, _inter(batched, H))
        flat = value.reshape(-1, H).contiguous()
        out = self.engine.expert_pairs(lw, flat, indices)
        return out.reshape(*indices.shape, H)


class StreamingSwitchGLU(StreamingExperts):
    """model._StreamingSwitchGLU over the fused w13 = [w3; w1] layout; the
    activation is silu(gate) * up, clamped when `swiglu_limit` > 0."""

    def __init__(self, layer: int, cache, engine: Engine, swiglu_limit: float = 0.0):
        super().__init__(layer, cache, engine)
        self.swiglu_limit = swiglu_limit

    def __call__(self, x: torch.Tensor, indices: torch.Tensor) -> torch.Tensor:
        batched = self.cache.current_batched(self.layer)
        H = x.shape[-1]
        lw = LayerWeights.from_batched(batched, H, _inter(batched, H), swiglu_limit=self.swiglu_limit)
        out = self.engine.expert_pairs(lw, x.reshape(-1, H).contiguous(), indices)
        return out.reshape(*indices.shape, H)


class SparseMoE:
    """qwen4_exp.SparseMoE: softmax top-k router (renormalised), sigmoid-gated
    shared expert and the weighted combine, in one library call."""

    def __init__(self, engine: Engine, layer: LayerWeights, top_k: int):
        self.engine, self.layer, self.top_k = engine, layer, top_k

    def route(self, value: torch.Tensor):
        """(scores fp32 [..., K] renormalised over the kept experts, indices int32 [..., K])."""
        H = value.shape[-1]
        w, idx = self.engine.route(self.layer, value.reshape(-1, H).contiguous(), self.top_k)
        return w.reshape(*value.shape[:-1], self.top_k), idx.reshape(*value.shape[:-1], self.top_k)

    def __call__(self, value: torch.Tensor, routes=None) -> torch.Tensor:
        H = value.shape[-1]
        flat = value.reshape(-1, H).contiguous()
        r = None if routes is None else tuple(t.reshape(flat.shape[0], self.top_k) for t in routes)
        out = self.engine.forward(self.layer, flat, self.top_k, routes=r)
        return out.reshape(value.shape)


class MoE(SparseMoE):
    """deepseek_v41.moe.MoE: sqrt-softplus gate with selection bias, weights
    / (sum + 1e-20) * route_scale, clamped SwiGLU, ungated shared expert."""


def streaming_moe(engine: Engine, layer: LayerWeights, x: torch.Tensor, top_k: int) -> torch.Tensor:
    """model._streaming_moe: gate -> shared -> routed -> route_reduce + shared."""
    H = x.shape[-1]
    return engine.forward(layer, x.reshape(-1, H).contiguous(), top_k).reshape(x.shape)


def _inter(batched, H: int) -> int:
    if isinstance(batched, QwenBatchedExperts):
        return batched.gate_up.shape[1] // 2
    if isinstance(batched, FP8BatchedExperts):
        return batched.w13.shape[1] // 2
    return batched.w13.shape[1] // 2
