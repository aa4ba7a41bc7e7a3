"""Expert blob layouts and the weight views handed to the expert kernels.

Mirrors runtime/deepseek_v4_ssd/expert_layout.py (region tables and
``batched_layer_layout``) and the view dataclasses of expert_cache.py:30-76,
with PyTorch tensors in place of MLX arrays.  The bytes are used in place:
an expert's projection is addressed as ``base + e * stride``.
"""
from __future__ import annotations

import bisect
from dataclasses import dataclass
from typing import NamedTuple

import torch

from . import lib


class Region(NamedTuple):
    """One tensor inside an expert blob (manifest.Tensor: name, dtype, shape, offset, length)."""
    name: str
    dtype: str
    shape: tuple[int, ...]
    offset: int
    length: int


def qwen_regions(H: int, I: int) -> dict[str, Region]:
    """Qwen blob: gate_up.weight | gate_up.scale | down.weight | down.scale
    (Sources/DeepSeekRepack/Qwen.swift:51-65; gate rows first)."""
    regs, off = {}, 0
    for name, dtype, shape, length in (
        ("gate_up.weight", "U32", (2 * I, H // 8), 2 * I * H // 2),
        ("gate_up.scale", "U8", (2 * I, H // 32), 2 * I * H // 32),
        ("down.weight", "U32", (H, I // 8), H * I // 2),
        ("down.scale", "U8", (H, I // 32), H * I // 32),
    ):
        regs[name] = Region(name, dtype, shape, off, length)
        off += length
    return regs


def fused_regions(H: int, I: int) -> dict[str, Region]:
    """DeepSeek / MiMo fused blob: w3 | w1 | w2 | w3.s | w1.s | w2.s with the
    virtual w13 = [w3; w1] (expert_layout.py:8-63)."""
    regs, off = {}, 0

    def add(name, dtype, shape, length):
        nonlocal off
        regs[name] = Region(name, dtype, shape, off, length)
        off += length

    add("w3.weight", "U32", (I, H // 8), I * H // 2)
    add("w1.weight", "U32", (I, H // 8), I * H // 2)
    add("w2.weight", "U32", (H, I // 8), H * I // 2)
    scale0 = off
    add("w3.scale", "U8", (I, H // 32), I * H // 32)
    add("w1.scale", "U8", (I, H // 32), I * H // 32)
    add("w2.scale", "U8", (H, I // 32), H * I // 32)
    regs["w13.weight"] = Region("w13.weight", "U32", (2 * I, H // 8), 0, I * H)
    regs["w13.scale"] = Region("w13.scale", "U8", (2 * I, H // 32), scale0, 2 * I * H // 32)
    return regs


def fp8_regions(H: int, I: int) -> dict[str, Region]:
    """FP8 E4M3 blob with fp32 128x128 block scales (new layout, up rows first):
    w13.weight | w2.weight | w13.scale | w2.scale."""
    regs, off = {}, 0
    for name, dtype, shape, length in (
        ("w13.weight", "F8_E4M3", (2 * I, H), 2 * I * H),
        ("w2.weight", "F8_E4M3", (H, I), H * I),
        ("w13.scale", "F32", (2 * I // 128, H // 128), 4 * (2 * I // 128) * (H // 128)),
        ("w2.scale", "F32", (H // 128, I // 128), 4 * (H // 128) * (I // 128)),
    ):
        regs[name] = Region(name, dtype, shape, off, length)
        off += length
    return regs


def blob_size(regions: dict[str, Region], batched: tuple[str, ...]) -> int:
    return sum(regions[n].length for n in batched)


def batched_layer_layout(regions: dict[str, Region], batched: tuple[str, ...], blob_size: int,
                         expert_count: int) -> dict[str, tuple[int, int, int]]:
    """Where every region of an expert blob lands in a region-major layer buffer.

    The layer buffer holds the `batched` regions one after another in blob
    order, each repeated for all `expert_count` experts, so every batched
    region is one contiguous [E, ...] array.  Returns name -> (base, stride,
    inner) for every region of `regions`: expert e's bytes of `name` start at
    base + e * stride + inner, where (base, stride) belong to the batched
    region that contains it.  This is the contract of the reference's
    batched_layer_layout (runtime/deepseek_v4_ssd/expert_layout.py:83-119);
    the batched regions must tile [0, blob_size) exactly."""
    tiles = sorted((regions[n].offset, regions[n].length, n) for n in batched)
    # tiling check: each batched region starts where the previous one ended
    cursor = 0
    for offset, length, name in tiles:
        if offset != cursor:
            raise ValueError(f"batched region {name} at byte {offset} leaves a gap or an overlap in the expert blob "
                             f"(expected byte {cursor})")
        cursor = offset + length
    if cursor != blob_size:
        raise ValueError(f"batched regions span {cursor} bytes of a {blob_size}-byte expert blob")
    # layer-buffer base of each tile: the tiles before it, each expert_count times
    ends = [offset + length for offset, length, _ in tiles]
    bases = [0] * len(tiles)
    for j in range(1, len(tiles)):
        bases[j] = bases[j - 1] + expert_count * tiles[j - 1][1]
    placed = {}
    for name, reg in regions.items():
        # the first tile (in blob order) whose end reaches this region's end
        j = bisect.bisect_left(ends, reg.offset + reg.length)
        if j == len(tiles) or tiles[j][0] > reg.offset:
            raise ValueError(f"region {name} does not lie inside one batched region")
        placed[name] = (bases[j], tiles[j][1], reg.offset - tiles[j][0])
    return placed


QWEN_BATCHED = ("gate_up.weight", "gate_up.scale", "down.weight", "down.scale")
FUSED_BATCHED = ("w13.weight", "w2.weight", "w13.scale", "w2.scale")
FP8_BATCHED = ("w13.weight", "w2.weight", "w13.scale", "w2.scale")


@dataclass(frozen=True)
class Projection:
    """One projection of every expert: expert e at weight.data_ptr() + e * weight_stride."""
    weight: torch.Tensor
    weight_stride: int
    scale: torch.Tensor
    scale_stride: int

    @staticmethod
    def stacked(weight: torch.Tensor, scale: torch.Tensor) -> "Projection":
        """From [E, ...] views whose per-expert slices are contiguous (the
        expert stride may exceed the slice: region-major layer buffers)."""
        for t in (weight, scale):
            if t.dim() < 2 or not t[0].is_contiguous():
                raise ValueError("each expert's projection must be one contiguous block")
        return Projection(weight, weight.stride(0) * weight.element_size(), scale,
                          scale.stride(0) * scale.element_size())

    def matrix(self) -> lib.Matrix:
        return lib.Matrix(self.weight.data_ptr(), self.weight_stride, self.scale.data_ptr(), self.scale_stride)


@dataclass(frozen=True)
class QwenExpertWeights:
    """One Qwen expert (expert_cache.py:63-68)."""
    gate_up: torch.Tensor
    gate_up_scales: torch.Tensor
    down: torch.Tensor
    down_scales: torch.Tensor


@dataclass(frozen=True)
class QwenBatchedExperts:
    """Every expert of a Qwen layer, [E, ...] views (expert_cache.py:71-76)."""
    gate_up: torch.Tensor
    gate_up_scales: torch.Tensor
    down: torch.Tensor
    down_scales: torch.Tensor


@dataclass(frozen=True)
class BatchedExperts:
    """Every expert of a DeepSeek / MiMo layer (expert_cache.py:51-60); w13 = [w3; w1]."""
    w1: torch.Tensor | None
    w1_scales: torch.Tensor | None
    w2: torch.Tensor
    w2_scales: torch.Tensor
    w3: torch.Tensor | None
    w3_scales: torch.Tensor | None
    w13: torch.Tensor | None = None
    w13_scales: torch.Tensor | None = None


@dataclass(frozen=True)
class FP8BatchedExperts:
    """Every expert of an FP8 E4M3 layer with fp32 128x128 block scales; w13 = [w3; w1]."""
    w13: torch.Tensor
    w13_scales: torch.Tensor
    w2: torch.Tensor
    w2_scales: torch.Tensor


def projections(batched) -> tuple[int, Projection, Projection]:
    """(layout, fused gate/up projection, down projection) of a batched view."""
    if isinstance(batched, QwenBatchedExperts):
        return (lib.LAYOUT_QWEN_GATE_UP_MXFP4, Projection.stacked(batched.gate_up, batched.gate_up_scales),
                Projection.stacked(batched.down, batched.down_scales))
    if isinstance(batched, FP8BatchedExperts):
        return (lib.LAYOUT_W13_FP8_B128, Projection.stacked(batched.w13, batched.w13_scales),
                Projection.stacked(batched.w2, batched.w2_scales))
    if isinstance(batched, BatchedExperts):
        if batched.w13 is None or batched.w13_scales is None:
            raise ValueError("the fused expert path needs the w13 = [w3; w1] view of the blob")
        return (lib.LAYOUT_DS_W13_MXFP4, Projection.stacked(batched.w13, batched.w13_scales),
                Projection.stacked(batched.w2, batched.w2_scales))
    raise TypeError(f"unsupported expert view {type(batched).__name__}")
