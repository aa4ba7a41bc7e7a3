"""ctypes binding of ``libwhallm_moe.so`` (declared in ``include/whallm_moe.h``).

The library is the only compute path: if it is missing or the GPU is not an
sm_100 part, every call raises -- there is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

# the in-tree build; WHALLM_MOE_LIB names another build of the same library
LIB_PATH = Path(os.environ.get("WHALLM_MOE_LIB") or Path(__file__).resolve().parent / "libwhallm_moe.so")

WM_OK, WM_ERROR, WM_CANCELLED = 0, 1, 2

LAYOUT_QWEN_GATE_UP_MXFP4, LAYOUT_DS_W13_MXFP4, LAYOUT_W13_FP8_B128, LAYOUT_W13_FP8_B32 = 0, 1, 2, 3
FORMAT_MXFP4, FORMAT_FP8_B128, FORMAT_FP8_B32 = 0, 1, 2
CONV_MLX, CONV_METAL = 0, 1
ROUTER_SOFTMAX, ROUTER_SQRTSOFTPLUS, ROUTER_SIGMOID, ROUTER_SIGMOID_GROUPED = 0, 1, 2, 3
SHARED_NONE, SHARED_SIGMOID_GATE, SHARED_ONE = 0, 1, 2
FLAG_SKIP_NEGATIVE_ROUTES = 1
FLAG_MMA_DECODE = 4
FLAG_F16_GEMM = 8
FLAG_SPLIT_SMALL_CALLS = 16
FLAG_FUSED_DECODE = 32

# Every entry point the header declares (checked by the CPU test suite).
EXPORTS = (
    "wm_create", "wm_destroy", "wm_error", "wm_sync", "wm_counters_get",
    "wm_dequant", "wm_route", "wm_expert_pairs", "wm_combine", "wm_ep_plan", "wm_moe_forward",
    "wm_profile_enable", "wm_profile_read", "wm_profile_reset",
    "wm_moe_forward_noalloc", "wm_moe_forward_noalloc_status",
    "wm_ep_create", "wm_ep_destroy", "wm_ep_ipc_handle", "wm_ep_open_peer", "wm_ep_buffer",
    "wm_ep_dispatch", "wm_ep_return", "wm_ep_wait", "wm_ep_experts",
)

_P = ctypes.c_void_p
_I32 = ctypes.c_int32
_I64 = ctypes.c_int64


class WMError(RuntimeError):
    """A failed library call (message from wm_error)."""


class Options(ctypes.Structure):
    _fields_ = [
        ("max_tokens", _I64), ("max_hidden", _I32), ("max_inter", _I32), ("max_experts", _I32),
        ("max_topk", _I32), ("gemv_max_tokens", _I32), ("flags", _I32),
    ]


class Matrix(ctypes.Structure):
    _fields_ = [("weight", _P), ("weight_stride", _I64), ("scale", _P), ("scale_stride", _I64)]


class MoeArgs(ctypes.Structure):
    _fields_ = [
        ("T", _I32), ("H", _I32), ("I", _I32), ("E", _I32), ("K", _I32),
        ("layout", _I32),
        ("w13", Matrix), ("w2", Matrix), ("shared_w13", Matrix), ("shared_w2", Matrix),
        ("shared_gate", _I32), ("shared_gate_weight", _P),
        ("x", _P),
        ("router", _I32), ("router_weight", _P), ("router_bias", _P),
        ("n_groups", _I32), ("topk_groups", _I32), ("route_scale", ctypes.c_float),
        ("routes_idx", _P), ("routes_w", _P),
        ("swiglu_limit", ctypes.c_float),
        ("out", _P), ("out_idx", _P), ("out_w", _P),
        ("norm_weight", _P), ("norm_eps", ctypes.c_float), ("x_norm", _P),
    ]


class Counters(ctypes.Structure):
    _fields_ = [
        ("calls_forward", _I64), ("calls_pairs", _I64), ("calls_route", _I64), ("calls_dequant", _I64),
        ("launches", _I64), ("gemv_calls", _I64), ("gemm_calls", _I64), ("decode_calls", _I64),
        ("bs_gemm_calls", _I64),
    ]


class ProfileEntry(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char * 32), ("launches", _I64), ("total_ms", ctypes.c_double)]


_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Load the library (raises if it was not built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise WMError(f"{LIB_PATH.name} is not built: run `python -m whallm_b200.build`")
    L = ctypes.CDLL(str(LIB_PATH))
    L.wm_create.argtypes = [_I32, ctypes.POINTER(Options), ctypes.c_char_p, ctypes.c_size_t]
    L.wm_create.restype = _P
    L.wm_destroy.argtypes = [_P]
    L.wm_destroy.restype = None
    L.wm_error.argtypes = [_P]
    L.wm_error.restype = ctypes.c_char_p
    L.wm_sync.argtypes = [_P, _P]
    L.wm_counters_get.argtypes = [_P, ctypes.POINTER(Counters)]
    L.wm_counters_get.restype = None
    L.wm_dequant.argtypes = [_P, _I32, _P, _P, _I64, _I64, _I32, _P, _P]
    L.wm_route.argtypes = [_P, ctypes.POINTER(MoeArgs), _P, _P, _P, _P]
    L.wm_expert_pairs.argtypes = [_P, ctypes.POINTER(MoeArgs), _P, _P]
    L.wm_moe_forward.argtypes = [_P, ctypes.POINTER(MoeArgs), _P]
    L.wm_combine.argtypes = [_P, _I64, _I32, _I32, _P, _P, _P, _P, _I32, _P, _P, _P, _P]
    L.wm_ep_plan.argtypes = [_P, _I64, _I32, _I32, _I32, _I32, _P, _P, _I32, _P, _P, _P, _P, _P]
    L.wm_profile_enable.argtypes = [_P, _I32]
    L.wm_profile_enable.restype = ctypes.c_int
    L.wm_profile_read.argtypes = [_P, ctypes.POINTER(ProfileEntry), _I32]
    L.wm_profile_read.restype = _I32
    L.wm_profile_reset.argtypes = [_P]
    L.wm_profile_reset.restype = None
    L.wm_moe_forward_noalloc.argtypes = [ctypes.POINTER(MoeArgs), _P, ctypes.c_char_p, ctypes.c_size_t]
    L.wm_moe_forward_noalloc.restype = ctypes.c_int
    L.wm_moe_forward_noalloc_status.argtypes = [_P, ctypes.c_char_p, ctypes.c_size_t]
    L.wm_moe_forward_noalloc_status.restype = ctypes.c_int
    L.wm_ep_create.argtypes = [_I32, _I32, _I32, _I64, _I32, ctypes.c_char_p, ctypes.c_size_t]
    L.wm_ep_create.restype = _P
    L.wm_ep_destroy.argtypes = [_P]
    L.wm_ep_destroy.restype = None
    L.wm_ep_ipc_handle.argtypes = [_P, _P]
    L.wm_ep_open_peer.argtypes = [_P, _I32, _P]
    L.wm_ep_buffer.argtypes = [_P, _I32]
    L.wm_ep_buffer.restype = _P
    L.wm_ep_dispatch.argtypes = [_P, _P, _I64, _I32, _I32, _P, _P, _P, _P]
    L.wm_ep_return.argtypes = [_P, _P, _P, _P]
    L.wm_ep_wait.argtypes = [_P, _P, _I32, _P]
    L.wm_ep_experts.argtypes = [_P, _P, ctypes.POINTER(MoeArgs), _P]
    for name in ("wm_sync", "wm_dequant", "wm_route", "wm_expert_pairs", "wm_combine", "wm_ep_plan",
                 "wm_moe_forward", "wm_ep_ipc_handle", "wm_ep_open_peer", "wm_ep_dispatch", "wm_ep_return",
                 "wm_ep_wait", "wm_ep_experts"):
        getattr(L, name).restype = ctypes.c_int
    _lib = L
    return L


class Context:
    """One library handle on one CUDA device, sized by its maxima."""

    def __init__(self, device: int = 0, *, max_tokens: int, max_hidden: int, max_inter: int, max_experts: int,
                 max_topk: int, gemv_max_tokens: int = 0, flags: int = 0):
        L = load()
        self._lib = L
        opt = Options(max_tokens=max_tokens, max_hidden=max_hidden, max_inter=max_inter,
                      max_experts=max_experts, max_topk=max_topk, gemv_max_tokens=gemv_max_tokens, flags=flags)
        err = ctypes.create_string_buffer(512)
        handle = L.wm_create(device, ctypes.byref(opt), err, len(err))
        if not handle:
            raise WMError(err.value.decode() or "wm_create failed")
        self.handle = handle
        self.device = device
        self.options = opt

    def close(self) -> None:
        if getattr(self, "handle", None):
            self._lib.wm_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def error(self) -> str:
        return self._lib.wm_error(self.handle).decode()

    def check(self, rc: int) -> None:
        if rc == WM_CANCELLED:
            raise WMError("cancelled")
        if rc != WM_OK:
            raise WMError(self.error())

    def sync(self, stream: int | None = None) -> None:
        self.check(self._lib.wm_sync(self.handle, stream))

    def counters(self) -> Counters:
        c = Counters()
        self._lib.wm_counters_get(self.handle, ctypes.byref(c))
        return c

    def profile(self, enable: bool) -> None:
        self.check(self._lib.wm_profile_enable(self.handle, 1 if enable else 0))

    def profile_read(self) -> dict[str, tuple[int, float]]:
        """kernel group -> (timed launches, total ms) since the last reset."""
        buf = (ProfileEntry * 16)()
        n = self._lib.wm_profile_read(self.handle, buf, 16)
        return {buf[i].name.decode(): (int(buf[i].launches), float(buf[i].total_ms)) for i in range(n)}

    def profile_reset(self) -> None:
        self._lib.wm_profile_reset(self.handle)

    def dequant(self, fmt: int, weight: int, scale: int, rows: int, cols: int, convention: int, out: int,
                stream: int | None) -> None:
        self.check(self._lib.wm_dequant(self.handle, fmt, weight, scale, rows, cols, convention, out, stream))

    def route(self, args: MoeArgs, logits: int | None, idx: int, w: int, stream: int | None) -> None:
        self.check(self._lib.wm_route(self.handle, ctypes.byref(args), logits, idx, w, stream))

    def expert_pairs(self, args: MoeArgs, routed: int, stream: int | None) -> None:
        self.check(self._lib.wm_expert_pairs(self.handle, ctypes.byref(args), routed, stream))

    def combine(self, T: int, H: int, K: int, pairs: int, pair_pos: int | None, w: int, shared: int | None,
                shared_gate: int, x: int | None, shared_gate_weight: int | None, out: int, stream: int | None) -> None:
        self.check(self._lib.wm_combine(self.handle, T, H, K, pairs, pair_pos, w, shared, shared_gate, x,
                                        shared_gate_weight, out, stream))

    def ep_plan(self, T: int, K: int, per_rank: int, world: int, capacity: int, idx: int, x: int, H: int,
                send_counts: int, pair_pos: int, send_eid: int, send_x: int, stream: int | None) -> None:
        self.check(self._lib.wm_ep_plan(self.handle, T, K, per_rank, world, capacity, idx, x, H, send_counts,
                                        pair_pos, send_eid, send_x, stream))

    def moe_forward(self, args: MoeArgs, stream: int | None) -> None:
        self.check(self._lib.wm_moe_forward(self.handle, ctypes.byref(args), stream))

    def ep_dispatch(self, ep: "EpBuffer", T: int, K: int, per_rank: int, idx: int, x: int, pair_pos: int,
                    stream: int | None) -> None:
        self.check(self._lib.wm_ep_dispatch(self.handle, ep.handle, T, K, per_rank, idx, x, pair_pos, stream))

    def ep_return(self, ep: "EpBuffer", y: int, stream: int | None) -> None:
        self.check(self._lib.wm_ep_return(self.handle, ep.handle, y, stream))

    def ep_wait(self, ep: "EpBuffer", which: int, stream: int | None) -> None:
        self.check(self._lib.wm_ep_wait(self.handle, ep.handle, which, stream))

    def ep_experts(self, ep: "EpBuffer", args: MoeArgs, stream: int | None) -> None:
        self.check(self._lib.wm_ep_experts(self.handle, ep.handle, ctypes.byref(args), stream))


class EpBuffer:
    """This rank's exchange buffer for expert-parallel exchanges over peer
    memory (wm_ep_*): recv_x / recv_e / back regions, mapped into the peers'
    address spaces through 64-byte CUDA IPC handles."""

    def __init__(self, device: int, world: int, rank: int, capacity: int, hidden: int):
        L = load()
        self._lib = L
        err = ctypes.create_string_buffer(512)
        handle = L.wm_ep_create(device, world, rank, capacity, hidden, err, len(err))
        if not handle:
            raise WMError(err.value.decode() or "wm_ep_create failed")
        self.handle = handle
        self.device, self.world, self.rank, self.capacity, self.hidden = device, world, rank, capacity, hidden

    def ipc_handle(self) -> bytes:
        buf = ctypes.create_string_buffer(64)
        if self._lib.wm_ep_ipc_handle(self.handle, buf) != WM_OK:
            raise WMError("cudaIpcGetMemHandle failed for the exchange buffer")
        return buf.raw

    def open_peer(self, peer: int, handle: bytes) -> None:
        buf = ctypes.create_string_buffer(bytes(handle), 64)
        if self._lib.wm_ep_open_peer(self.handle, peer, buf) != WM_OK:
            raise WMError(f"cudaIpcOpenMemHandle failed for the exchange buffer of rank {peer}")

    def buffer(self, which: int) -> int:
        return int(self._lib.wm_ep_buffer(self.handle, which))

    def close(self) -> None:
        if getattr(self, "handle", None):
            self._lib.wm_ep_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
