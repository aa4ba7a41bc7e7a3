"""Host-side (token, expert) pair scheduling.

``expert_waves`` keeps the contract of the reference's pure-numpy scheduler
(runtime/deepseek_v4_ssd/qwen_expert_waves.py:23-51): every flattened pair is
visited once, grouped by expert in stable order, at most ``capacity`` experts
per wave.  On B200 every expert of a layer is resident in HBM, so the device
plan (csrc/wm_plan.cu) forms all groups in one pass with no waves; callers
that still stream experts through a bounded slot pool use this function.

``sorted_rows`` states the device plan's row order in numpy: the pairs of
expert e occupy rows [offsets[e], offsets[e] + counts[e]) in ascending
(token, k) order, each group starting on an `align`-row boundary, and the
shared expert (index E, when present) takes one row per token after them.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Iterator

import numpy as np


@dataclass(frozen=True)
class ExpertWave:
    """One wave: (expert id, positions into the flattened routes) per expert,
    experts ascending, positions ascending within an expert."""
    groups: tuple[tuple[int, np.ndarray], ...]

    @property
    def expert_ids(self) -> tuple[int, ...]:
        return tuple(g[0] for g in self.groups)


def _count_arg(value, what: str) -> int:
    # plain ints only: bools, floats and numpy scalars are refused, as the reference does
    if isinstance(value, bool) or not isinstance(value, int) or value <= 0:
        raise ValueError(f"{what} must be a positive integer, got {value!r}")
    return value


def _flat_routes(indices, expert_count: int) -> np.ndarray:
    routes = np.asarray(indices).reshape(-1)
    if routes.size and routes.dtype.kind not in "iu":
        raise ValueError(f"routes must hold integer expert ids, not {routes.dtype}")
    if routes.size and (routes.min() < 0 or routes.max() >= expert_count):
        raise ValueError(f"an expert id lies outside [0, {expert_count})")
    return routes


def expert_waves(indices, capacity: int, expert_count: int) -> Iterator[ExpertWave]:
    """Visit every flattened routing pair exactly once, in stable expert order,
    at most `capacity` experts per wave; positions index the flattened routes."""
    _count_arg(capacity, "wave capacity")
    _count_arg(expert_count, "expert count")
    flat = _flat_routes(indices, expert_count)
    if flat.size == 0:
        return
    # counting sort: bucket sizes, then positions in ascending order per bucket
    counts = np.bincount(flat, minlength=expert_count)
    order = np.argsort(flat, kind="stable")
    present = np.flatnonzero(counts)
    bounds = np.concatenate([[0], np.cumsum(counts[present])])
    wave: list[tuple[int, np.ndarray]] = []
    for j, expert in enumerate(present):
        wave.append((int(expert), order[bounds[j]:bounds[j + 1]]))
        if len(wave) == capacity:
            yield ExpertWave(tuple(wave))
            wave = []
    if wave:
        yield ExpertWave(tuple(wave))


def sorted_rows(indices: np.ndarray, expert_count: int, has_shared: bool = False, align: int = 1):
    """(counts [E+1], offsets [E+2], pair_pos [T*K], row_token [rows]) of the device plan."""
    idx = np.asarray(indices).reshape(indices.shape[0], -1)
    T, K = idx.shape
    E = expert_count
    counts = np.zeros(E + 1, np.int64)
    counts[:E] = np.bincount(idx.reshape(-1), minlength=E)[:E]
    counts[E] = T if has_shared else 0
    padded = (counts + align - 1) // align * align
    offsets = np.concatenate([[0], np.cumsum(padded)])
    pair_pos = np.empty(T * K, np.int64)
    row_token = np.full(offsets[-1], -1, np.int64)
    run = offsets[:E].copy()
    for t in range(T):
        for k in range(K):
            e = idx[t, k]
            pair_pos[t * K + k] = run[e]
            row_token[run[e]] = t
            run[e] += 1
    if has_shared:
        row_token[offsets[E]:offsets[E] + T] = np.arange(T)
    return counts, offsets, pair_pos, row_token
