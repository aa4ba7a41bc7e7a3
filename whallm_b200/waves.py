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
    groups: tuple[tuple[int, np.ndarray], ...]

    @property
    def expert_ids(self) -> tuple[int, ...]:
        return tuple(expert for expert, _ in self.groups)


def expert_waves(indices, capacity: int, expert_count: int) -> Iterator[ExpertWave]:
    """Visit every flattened routing pair exactly once, in stable expert order,
    at most `capacity` experts per wave; positions index the flattened routes."""
    if type(capacity) is not int or capacity < 1:
        raise ValueError("expert wave capacity must be a positive integer")
    if type(expert_count) is not int or expert_count < 1:
        raise ValueError("expert count must be a positive integer")
    selected = np.asarray(indices)
    if selected.size == 0:
        return
    if not np.issubdtype(selected.dtype, np.integer):
        raise ValueError("expert IDs must be integers")
    flat = selected.reshape(-1)
    if np.any(flat < 0) or np.any(flat >= expert_count):
        raise ValueError("expert ID is outside the model")
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
