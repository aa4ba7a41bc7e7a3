"""CPU oracle for the MoE expert-FFN path (TEST INFRASTRUCTURE ONLY).

A ctypes front end to ``wm_oracle.c``, the C restatement of Whallm's own
arithmetic for this path (each C function cites the reference file:line it
follows).  Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s
CPU-baseline / reference arm import this package; the product
(``whallm_b200``) never does, and fails loudly when its CUDA library is
missing instead of falling back here.

Pinned by: the Swift known-answer vectors of the reference's MXFP4 quantiser
(``tests/golden/mxfp4_kat.json``), the pure-numpy reference scheduler
``qwen_expert_waves.py`` run here (``tests/golden/expert_waves.json``) and
hand-checkable format identities.  The routed-expert maths behind
``mx.gather_qmm`` (mlx 0.32.2) is not installable here, so layer outputs are
checked against this restatement under the stated bf16 tolerance.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libwm_oracle.so"

CONV_MLX, CONV_METAL = 0, 1
LAYOUT_QWEN_GATE_UP_MXFP4, LAYOUT_DS_W13_MXFP4, LAYOUT_W13_FP8_B128, LAYOUT_W13_FP8_B32 = 0, 1, 2, 3
ROUTER_SOFTMAX, ROUTER_SQRTSOFTPLUS, ROUTER_SIGMOID, ROUTER_SIGMOID_GROUPED = 0, 1, 2, 3
SHARED_NONE, SHARED_SIGMOID_GATE, SHARED_ONE = 0, 1, 2
NUMERICS_BF16, NUMERICS_FP32 = 0, 1

_lib = None


def build() -> Path:
    """Compile the oracle with its Makefile (gcc + OpenMP)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        _lib = ctypes.CDLL(str(LIB_PATH))
        _declare(_lib)
    return _lib


P = ctypes.c_void_p
I64 = ctypes.c_int64
I32 = ctypes.c_int32
F32 = ctypes.c_float


class WmoExpert(ctypes.Structure):
    _fields_ = [("layout", I32), ("w13", P), ("w13_scale", P), ("w2", P), ("w2_scale", P)]


class WmoLayer(ctypes.Structure):
    _fields_ = [
        ("T", I64), ("H", I64), ("I", I64), ("E", I64), ("K", I64),
        ("layout", I32),
        ("w13", P), ("w13_stride", I64), ("w13_scale", P), ("w13_scale_stride", I64),
        ("w2", P), ("w2_stride", I64), ("w2_scale", P), ("w2_scale_stride", I64),
        ("sh_w13", P), ("sh_w13_scale", P), ("sh_w2", P), ("sh_w2_scale", P),
        ("shared_gate_kind", I32), ("shared_gate_weight", P),
        ("swiglu_limit", F32), ("numerics", I32), ("convention", I32),
    ]


def _declare(L: ctypes.CDLL) -> None:
    L.wmo_e2m1.argtypes, L.wmo_e2m1.restype = [ctypes.c_uint32, ctypes.c_int], F32
    L.wmo_e8m0.argtypes, L.wmo_e8m0.restype = [ctypes.c_uint32, ctypes.c_int], F32
    L.wmo_e4m3.argtypes, L.wmo_e4m3.restype = [ctypes.c_uint32], F32
    L.wmo_f32_to_bf16.argtypes, L.wmo_f32_to_bf16.restype = [F32], ctypes.c_uint16
    L.wmo_dequant_mxfp4.argtypes = [P, P, I64, I64, ctypes.c_int, P]
    L.wmo_dequant_fp8_b128.argtypes = [P, P, I64, I64, P]
    L.wmo_dequant_fp8_b32.argtypes = [P, P, I64, I64, P]
    L.wmo_quantize_bf16_mxfp4.argtypes = [P, I64, I64, P, P]
    L.wmo_quantize_fp8_mxfp4.argtypes = [P, P, I64, I64, P, P]
    L.wmo_expert_ffn.argtypes = [ctypes.POINTER(WmoExpert), I64, I64, P, I64, F32, ctypes.c_int, ctypes.c_int, P]
    L.wmo_linear.argtypes = [I32, P, P, I64, I64, P, I64, ctypes.c_int, P]
    L.wmo_router_logits.argtypes = [P, P, I64, I64, I64, P]
    L.wmo_router_logits.restype = None
    L.wmo_route.argtypes = [ctypes.c_int, P, P, I64, I64, I64, I64, I64, F32, P, P]
    L.wmo_route.restype = None
    L.wmo_moe_forward.argtypes = [ctypes.POINTER(WmoLayer), P, P, P, P, I64, P]
    L.wmo_expert_pairs.argtypes = [ctypes.POINTER(WmoLayer), P, P, P]
    L.wmo_max_threads.restype = ctypes.c_int
    L.wmo_set_threads.argtypes = [ctypes.c_int]
    L.wmo_set_threads.restype = None


def _p(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data_as(ctypes.c_void_p)


# ---------------------------------------------------------------- scalar formats

def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(values: np.ndarray) -> np.ndarray:
    """Round to nearest even (NaN kept quiet), as bits."""
    u = np.ascontiguousarray(values, dtype=np.float32).view(np.uint32)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(nan, ((u >> 16) | 0x40).astype(np.uint16), r)


def e2m1(code: int, convention: int = CONV_MLX) -> float:
    return lib().wmo_e2m1(code, convention)


def e8m0(byte: int, convention: int = CONV_MLX) -> float:
    return lib().wmo_e8m0(byte, convention)


def e4m3(byte: int) -> float:
    return lib().wmo_e4m3(byte)


# ---------------------------------------------------------------- dequant / quantise

def dequant_mxfp4(w: np.ndarray, s: np.ndarray, convention: int = CONV_MLX) -> np.ndarray:
    """Packed [rows, cols/2] + E8M0 [rows, cols/32] -> bf16 bits [rows, cols]."""
    w = np.ascontiguousarray(w, dtype=np.uint8)
    s = np.ascontiguousarray(s, dtype=np.uint8)
    rows, cols = w.shape[0], w.shape[1] * 2
    out = np.empty((rows, cols), np.uint16)
    if lib().wmo_dequant_mxfp4(_p(w), _p(s), rows, cols, convention, _p(out)):
        raise ValueError("MXFP4 columns must be a multiple of 32")
    return out


def dequant_fp8_b128(w: np.ndarray, s: np.ndarray) -> np.ndarray:
    w = np.ascontiguousarray(w, dtype=np.uint8)
    s = np.ascontiguousarray(s, dtype=np.float32)
    out = np.empty(w.shape, np.uint16)
    if lib().wmo_dequant_fp8_b128(_p(w), _p(s), w.shape[0], w.shape[1], _p(out)):
        raise ValueError("FP8 checkpoint contains reserved NaN codes or invalid block scales")
    return out


def dequant_fp8_b32(w: np.ndarray, s: np.ndarray) -> np.ndarray:
    w = np.ascontiguousarray(w, dtype=np.uint8)
    s = np.ascontiguousarray(s, dtype=np.uint8)
    out = np.empty(w.shape, np.uint16)
    lib().wmo_dequant_fp8_b32(_p(w), _p(s), w.shape[0], w.shape[1], _p(out))
    return out


def quantize_bf16_mxfp4(bits: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    bits = np.ascontiguousarray(bits, dtype=np.uint16)
    rows, cols = bits.shape
    w = np.empty((rows, cols // 2), np.uint8)
    s = np.empty((rows, cols // 32), np.uint8)
    if lib().wmo_quantize_bf16_mxfp4(_p(bits), rows, cols, _p(w), _p(s)):
        raise ValueError("MXFP4 source must contain complete BF16 rows")
    return w, s


def quantize_fp8_mxfp4(src: np.ndarray, inv_scales_bf16: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    src = np.ascontiguousarray(src, dtype=np.uint8)
    inv = np.ascontiguousarray(inv_scales_bf16, dtype=np.uint16)
    rows, cols = src.shape
    w = np.empty((rows, cols // 2), np.uint8)
    s = np.empty((rows, cols // 32), np.uint8)
    if lib().wmo_quantize_fp8_mxfp4(_p(src), _p(inv), rows, cols, _p(w), _p(s)):
        raise ValueError("MXFP4 FP8 source must contain complete 128 by 128 scale blocks")
    return w, s


# ---------------------------------------------------------------- experts, routers, layer

def linear(layout: int, w: np.ndarray, scale: np.ndarray, x_bits: np.ndarray, convention: int = CONV_MLX) -> np.ndarray:
    """y = x @ dequant(w).T as fp32 (double accumulation)."""
    x_bits = np.ascontiguousarray(x_bits, dtype=np.uint16)
    rows, kd = x_bits.shape
    O = w.shape[0]
    out = np.empty((rows, O), np.float32)
    lib().wmo_linear(layout, _p(np.ascontiguousarray(w)), _p(np.ascontiguousarray(scale)), O, kd, _p(x_bits), rows,
                     convention, _p(out))
    return out


def rms_norm(x_bits: np.ndarray, w_bits: np.ndarray, eps: float) -> np.ndarray:
    """Pre-MoE RMSNorm as bf16 bits [T, H]: bf16((x * r) * w) in fp32 with
    r = 1 / sqrt(mean(x^2) + eps) -- rms_norm_tg (DeepSeekNative/kernels.metal:443-465)
    and the float32 branch of GroupRMSNorm (qwen4_exp.py:93-117).  The sum of
    squares is taken in float64 here, so r can differ from a float32 sum in the
    last place."""
    x = bf16_to_f32(np.ascontiguousarray(x_bits, dtype=np.uint16))
    w = bf16_to_f32(np.ascontiguousarray(w_bits, dtype=np.uint16))
    ms = np.mean(np.square(x.astype(np.float64)), axis=-1, keepdims=True).astype(np.float32)
    r = (np.float32(1.0) / np.sqrt(ms + np.float32(eps))).astype(np.float32)
    return f32_to_bf16((x * r) * w)


def router_logits(x_bits: np.ndarray, w_bits: np.ndarray) -> np.ndarray:
    x_bits = np.ascontiguousarray(x_bits, dtype=np.uint16)
    w_bits = np.ascontiguousarray(w_bits, dtype=np.uint16)
    T, H = x_bits.shape
    E = w_bits.shape[0]
    out = np.empty((T, E), np.float32)
    lib().wmo_router_logits(_p(x_bits), _p(w_bits), T, H, E, _p(out))
    return out


def route(router: int, logits: np.ndarray, K: int, bias: np.ndarray | None = None, n_groups: int = 1,
          topk_groups: int = 1, route_scale: float = 1.0) -> tuple[np.ndarray, np.ndarray]:
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    T, E = logits.shape
    idx = np.empty((T, K), np.int32)
    w = np.empty((T, K), np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    lib().wmo_route(router, _p(logits), _p(b), T, E, K, n_groups, topk_groups, route_scale, _p(idx), _p(w))
    return idx, w


class Layer:
    """Numpy-side description of one MoE layer for the oracle.

    Routed experts are given per projection as [E, ...] arrays (weights and
    scales); the shared expert (optional) as single-expert arrays.
    """

    def __init__(self, layout: int, H: int, I: int, w13, w13_scale, w2, w2_scale, shared=None,
                 shared_gate_kind: int = SHARED_NONE, shared_gate_weight=None, swiglu_limit: float = 0.0,
                 numerics: int = NUMERICS_BF16, convention: int = CONV_MLX):
        self.layout, self.H, self.I = layout, H, I
        self.w13 = np.ascontiguousarray(w13)
        self.w13_scale = np.ascontiguousarray(w13_scale)
        self.w2 = np.ascontiguousarray(w2)
        self.w2_scale = np.ascontiguousarray(w2_scale)
        self.E = self.w13.shape[0]
        self.shared = None if shared is None else tuple(np.ascontiguousarray(a) for a in shared)
        self.shared_gate_kind = shared_gate_kind
        self.shared_gate_weight = None if shared_gate_weight is None else np.ascontiguousarray(
            shared_gate_weight, dtype=np.uint16)
        self.swiglu_limit, self.numerics, self.convention = swiglu_limit, numerics, convention

    def _struct(self, T: int, K: int) -> WmoLayer:
        s = WmoLayer()
        s.T, s.H, s.I, s.E, s.K = T, self.H, self.I, self.E, K
        s.layout = self.layout
        s.w13, s.w13_stride = _p(self.w13), self.w13[0].nbytes
        s.w13_scale, s.w13_scale_stride = _p(self.w13_scale), self.w13_scale[0].nbytes
        s.w2, s.w2_stride = _p(self.w2), self.w2[0].nbytes
        s.w2_scale, s.w2_scale_stride = _p(self.w2_scale), self.w2_scale[0].nbytes
        if self.shared is not None:
            s.sh_w13, s.sh_w13_scale, s.sh_w2, s.sh_w2_scale = (_p(a) for a in self.shared)
        s.shared_gate_kind = self.shared_gate_kind
        s.shared_gate_weight = _p(self.shared_gate_weight)
        s.swiglu_limit, s.numerics, s.convention = self.swiglu_limit, self.numerics, self.convention
        return s

    def forward(self, x_bits: np.ndarray, idx: np.ndarray, w: np.ndarray, tokens: np.ndarray | None = None) -> np.ndarray:
        """Combined output bits [T, H]; with ``tokens``, only those rows are computed (others 0)."""
        x_bits = np.ascontiguousarray(x_bits, dtype=np.uint16)
        idx = np.ascontiguousarray(idx, dtype=np.int32)
        w = np.ascontiguousarray(w, dtype=np.float32)
        T, K = idx.shape
        out = np.zeros((T, self.H), np.uint16)
        st = self._struct(T, K)
        only = None if tokens is None else np.ascontiguousarray(tokens, dtype=np.int32)
        # wmo_moe_forward takes int32 token ids for the subset
        rc = lib().wmo_moe_forward(ctypes.byref(st), _p(x_bits), _p(idx), _p(w), _p(only),
                                   0 if only is None else only.size, _p(out))
        if rc == 2:
            raise ValueError("expert ID is outside the model")
        if rc:
            raise MemoryError("oracle allocation failed")
        return out

    def pairs(self, x_bits: np.ndarray, idx: np.ndarray) -> np.ndarray:
        """Routed rows [T, K, H] (bf16 bits) without the combine."""
        x_bits = np.ascontiguousarray(x_bits, dtype=np.uint16)
        idx = np.ascontiguousarray(idx, dtype=np.int32)
        T, K = idx.shape
        out = np.zeros((T, K, self.H), np.uint16)
        st = self._struct(T, K)
        if lib().wmo_expert_pairs(ctypes.byref(st), _p(x_bits), _p(idx), _p(out)):
            raise MemoryError("oracle allocation failed")
        return out


def max_threads() -> int:
    return int(lib().wmo_max_threads())


def set_threads(n: int) -> None:
    """OpenMP threads of the oracle's later calls from this thread."""
    lib().wmo_set_threads(int(n))


def max_rel_error(y: np.ndarray, ref: np.ndarray) -> float:
    """max|y - ref| / max|ref| (both float arrays)."""
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    denom = np.max(np.abs(ref))
    return float(np.max(np.abs(y - ref)) / (denom if denom > 0 else 1.0))
