"""Seeded synthetic MoE layers with the shapes and value distributions of the
benchmark configurations (no checkpoints or datasets are used anywhere).

  config 0  one SwiGLU expert, H=2048, I=512, MXFP4, 4 tokens
  config 1  decode: 512 experts (I=512) + 1 shared, top-10 softmax, B = 1 / 8 / 64
  config 2  prefill: config-1 layer, 16384 tokens, Zipf(1.1) expert popularity
  config 3  DeepSeek-style FP8 E4M3 (fp32 128x128 block scales), H=7168,
            256 experts (I=2048) + shared, top-8 sigmoid group-limited (8 / 4), 8192 tokens
  config 4  8 stacked MXFP4 layers, H=7168, 384 experts (I=2048) + shared, top-8,
            256 decode + 4096 prefill tokens, uniform routing

MXFP4 bytes are uniform (so each E2M1 nibble is uniform over its 16 codes);
E8M0 scale bytes are 127 + U{-8..-2}; FP8 codes are uniform over the 254
finite E4M3 codes with block scales 2^U(-10, -4); activations are N(0, 1) in
bf16; router weights are N(0, 1/sqrt(H)) so logits are about N(0, 1).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from . import lib
from .layout import Projection
from .moe import LayerWeights, RouterWeights, SharedExpert


def _gen(seed: int, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def mxfp4_projection(E: int, rows: int, cols: int, g: torch.Generator, device, exp_lo: int = -8,
                     exp_hi: int = -2) -> tuple[torch.Tensor, torch.Tensor]:
    """Packed E2M1 [E, rows, cols/2] uint8 + E8M0 [E, rows, cols/32] uint8."""
    w = torch.randint(0, 256, (E, rows, cols // 2), generator=g, device=device, dtype=torch.uint8)
    s = (127 + torch.randint(exp_lo, exp_hi + 1, (E, rows, cols // 32), generator=g, device=device,
                             dtype=torch.int16)).to(torch.uint8)
    return w, s


def fp8_projection(E: int, rows: int, cols: int, g: torch.Generator, device) -> tuple[torch.Tensor, torch.Tensor]:
    """E4M3 [E, rows, cols] uint8 over the finite codes + fp32 [E, rows/128, cols/128] scales."""
    r = torch.randint(0, 254, (E, rows, cols), generator=g, device=device, dtype=torch.int16)
    w = torch.where(r < 127, r, r + 1).to(torch.uint8)  # skips 0x7F and 0xFF
    u = torch.rand((E, rows // 128, cols // 128), generator=g, device=device, dtype=torch.float32)
    s = torch.exp2(-10.0 + 6.0 * u)
    return w, s


def fp8_b32_projection(E: int, rows: int, cols: int, g: torch.Generator, device) -> tuple[torch.Tensor, torch.Tensor]:
    """E4M3 [E, rows, cols] over the finite codes + UE8M0 [E, rows/32, cols/32] scale bytes 127 + U{-10..-4}."""
    r = torch.randint(0, 254, (E, rows, cols), generator=g, device=device, dtype=torch.int16)
    w = torch.where(r < 127, r, r + 1).to(torch.uint8)
    s = (127 + torch.randint(-10, -3, (E, rows // 32, cols // 32), generator=g, device=device,
                             dtype=torch.int16)).to(torch.uint8)
    return w, s


def projection_for(layout: int):
    """The generator of a layout's projections (weights + scales)."""
    return {lib.LAYOUT_W13_FP8_B128: fp8_projection, lib.LAYOUT_W13_FP8_B32: fp8_b32_projection}.get(
        layout, mxfp4_projection)


def activations(T: int, H: int, g: torch.Generator, device) -> torch.Tensor:
    return torch.randn((T, H), generator=g, device=device, dtype=torch.float32).to(torch.bfloat16)


@dataclass
class Workload:
    layer: LayerWeights
    x: torch.Tensor
    K: int
    name: str


def qwen_layer(E: int = 512, H: int = 2048, I: int = 512, device="cuda", seed: int = 0, shared: bool = True,
               router: bool = True, zipf_s: float = 0.0) -> LayerWeights:
    """Config-1/2 layer: Qwen gate_up/down MXFP4 blobs, softmax router, sigmoid-gated shared expert.

    With zipf_s > 0 the router gets a logit bias -zipf_s * ln(1 + pi(e)) (pi a
    seeded permutation), so expert popularity follows Zipf(zipf_s)."""
    g = _gen(seed, device)
    w13, s13 = mxfp4_projection(E, 2 * I, H, g, device)
    w2, s2 = mxfp4_projection(E, H, I, g, device)
    sh = None
    if shared:
        a, b = mxfp4_projection(1, 2 * I, H, g, device)
        c, d = mxfp4_projection(1, H, I, g, device)
        gate = (torch.randn((H,), generator=g, device=device) / math.sqrt(H)).to(torch.bfloat16)
        sh = SharedExpert(Projection.stacked(a, b), Projection.stacked(c, d), lib.SHARED_SIGMOID_GATE, gate)
    rw = None
    if router:
        wr = (torch.randn((E, H), generator=g, device=device) / math.sqrt(H)).to(torch.bfloat16)
        bias = None
        if zipf_s > 0:
            perm = torch.randperm(E, generator=g, device=device).to(torch.float32)
            bias = (-zipf_s * torch.log1p(perm)).to(torch.float32)
        rw = RouterWeights(wr, lib.ROUTER_SOFTMAX, bias)
    return LayerWeights(lib.LAYOUT_QWEN_GATE_UP_MXFP4, H, I, E, Projection.stacked(w13, s13),
                        Projection.stacked(w2, s2), shared=sh, router=rw)


def deepseek_fp8_layer(E: int = 256, H: int = 7168, I: int = 2048, device="cuda", seed: int = 0,
                       shared: bool = True, n_groups: int = 8, topk_groups: int = 4,
                       route_scale: float = 1.0) -> LayerWeights:
    """Config-3 layer: FP8 E4M3 w13 = [w3; w1] / w2 with fp32 128x128 scales,
    sigmoid group-limited router, ungated shared expert."""
    g = _gen(seed, device)
    w13, s13 = fp8_projection(E, 2 * I, H, g, device)
    w2, s2 = fp8_projection(E, H, I, g, device)
    sh = None
    if shared:
        a, b = fp8_projection(1, 2 * I, H, g, device)
        c, d = fp8_projection(1, H, I, g, device)
        sh = SharedExpert(Projection.stacked(a, b), Projection.stacked(c, d), lib.SHARED_ONE)
    wr = (torch.randn((E, H), generator=g, device=device) / math.sqrt(H)).to(torch.bfloat16)
    rw = RouterWeights(wr, lib.ROUTER_SIGMOID_GROUPED, None, n_groups, topk_groups, route_scale)
    return LayerWeights(lib.LAYOUT_W13_FP8_B128, H, I, E, Projection.stacked(w13, s13), Projection.stacked(w2, s2),
                        shared=sh, router=rw)


def deepseek_mxfp4_layer(E: int = 384, H: int = 7168, I: int = 2048, device="cuda", seed: int = 0,
                         shared: bool = True, swiglu_limit: float = 0.0) -> LayerWeights:
    """Config-4 layer: fused w13 = [w3; w1] MXFP4 blobs, sigmoid router (no
    grouping, no bias: uniform routing), ungated shared expert."""
    g = _gen(seed, device)
    w13, s13 = mxfp4_projection(E, 2 * I, H, g, device)
    w2, s2 = mxfp4_projection(E, H, I, g, device)
    sh = None
    if shared:
        a, b = mxfp4_projection(1, 2 * I, H, g, device)
        c, d = mxfp4_projection(1, H, I, g, device)
        sh = SharedExpert(Projection.stacked(a, b), Projection.stacked(c, d), lib.SHARED_ONE)
    wr = (torch.randn((E, H), generator=g, device=device) / math.sqrt(H)).to(torch.bfloat16)
    rw = RouterWeights(wr, lib.ROUTER_SIGMOID)
    return LayerWeights(lib.LAYOUT_DS_W13_MXFP4, H, I, E, Projection.stacked(w13, s13), Projection.stacked(w2, s2),
                        shared=sh, router=rw, swiglu_limit=swiglu_limit)


def config(n: int, device="cuda", seed: int = 0, batch: int = 64) -> Workload:
    if n == 0:
        layer = qwen_layer(E=1, device=device, seed=seed, shared=False, router=False)
        return Workload(layer, activations(4, 2048, _gen(seed + 1, device), device), 1, "config0")
    if n == 1:
        layer = qwen_layer(device=device, seed=seed)
        return Workload(layer, activations(batch, 2048, _gen(seed + 1, device), device), 10, f"config1-b{batch}")
    if n == 2:
        layer = qwen_layer(device=device, seed=seed, zipf_s=1.1)
        return Workload(layer, activations(16384, 2048, _gen(seed + 1, device), device), 10, "config2")
    if n == 3:
        layer = deepseek_fp8_layer(device=device, seed=seed)
        return Workload(layer, activations(8192, 7168, _gen(seed + 1, device), device), 8, "config3")
    if n == 4:
        # one layer of the config-4 stack: 256 decode tokens and a 4096-token prefill chunk in one call
        layer = deepseek_mxfp4_layer(device=device, seed=seed)
        return Workload(layer, activations(256 + 4096, 7168, _gen(seed + 1, device), device), 8, "config4-layer")
    raise ValueError(f"no single-layer workload for config {n}")
