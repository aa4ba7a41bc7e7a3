"""Bridges the product's torch-side layer description to the oracle (test
infrastructure: copies the weights a check needs to the host)."""
from __future__ import annotations

import numpy as np
import torch

from . import SHARED_NONE, Layer


def bits(t: torch.Tensor) -> np.ndarray:
    """bf16 tensor -> uint16 bit array on the host."""
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def from_layer(layer, experts: list[int] | None = None, numerics: int = 0) -> Layer:
    """An oracle Layer over the experts of `layer` (a whallm_b200.moe.LayerWeights).

    With `experts`, only those expert slots are copied, in that order; routes
    must then name positions in that list."""

    def sub(t: torch.Tensor) -> np.ndarray:
        if experts is not None:
            t = t[torch.as_tensor(experts, device=t.device, dtype=torch.long)]
        return t.contiguous().cpu().numpy()

    shared, sgk, sgw = None, SHARED_NONE, None
    if layer.shared is not None:
        shared = tuple(a[0].contiguous().cpu().numpy() for a in (
            layer.shared.w13.weight, layer.shared.w13.scale, layer.shared.w2.weight, layer.shared.w2.scale))
        sgk = layer.shared.gate
        sgw = None if layer.shared.gate_weight is None else bits(layer.shared.gate_weight)
    return Layer(layer.layout, layer.H, layer.I, sub(layer.w13.weight), sub(layer.w13.scale),
                 sub(layer.w2.weight), sub(layer.w2.scale), shared=shared, shared_gate_kind=sgk,
                 shared_gate_weight=sgw, swiglu_limit=layer.swiglu_limit, numerics=numerics)
