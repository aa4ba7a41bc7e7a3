"""Host scheduling mirror against outputs of the reference's own scheduler (no GPU)."""
import json
from pathlib import Path

import numpy as np
import pytest

from whallm_b200.waves import expert_waves, sorted_rows

GOLDEN = Path(__file__).resolve().parent / "golden"


def test_expert_waves_match_reference_outputs():
    """qwen_expert_waves.py:23-51 run on seeded routes (tests/golden/expert_waves.json)."""
    data = json.loads((GOLDEN / "expert_waves.json").read_text())
    for case in data["cases"]:
        sel = np.array(case["selected"], np.int32)
        got = [[[e, pos.tolist()] for e, pos in w.groups] for w in expert_waves(sel, case["capacity"], case["experts"])]
        assert got == case["waves"]


def test_random_pair_coverage_order_and_capacity():
    """The invariants of the reference's portable tests (test_qwen_flash_portable.py:33-50)."""
    rng = np.random.default_rng(20260921)
    for tokens in (1, 2, 17, 128):
        selected = rng.integers(0, 512, size=(1, tokens, 10), dtype=np.int32)
        for capacity in (1, 10, 512, 1024):
            visited, ids = [], []
            for wave in expert_waves(selected, capacity, 512):
                assert len(wave.groups) <= capacity
                for expert, positions in wave.groups:
                    assert np.all(selected.reshape(-1)[positions] == expert)
                    assert np.all(np.diff(positions) > 0)
                    visited.extend(positions)
                    ids.append(expert)
            np.testing.assert_array_equal(np.sort(visited), np.arange(selected.size))
            assert ids == sorted(set(selected.reshape(-1)))


def test_empty_repeated_and_invalid_routes():
    assert list(expert_waves(np.empty((0, 10), dtype=int), 1, 512)) == []
    result = list(expert_waves(np.full((9, 10), 5), 1, 512))
    assert len(result) == 1
    np.testing.assert_array_equal(result[0].groups[0][1], np.arange(90))
    for capacity in (0, -1, True, 2.0):
        with pytest.raises(ValueError):
            list(expert_waves(np.array([0]), capacity, 512))
    for count in (0, -1, True, 1.0):
        with pytest.raises(ValueError):
            list(expert_waves(np.array([0]), 1, count))
    for ids in ([-1], [512], [1.2]):
        with pytest.raises(ValueError):
            list(expert_waves(np.asarray(ids), 2, 512))


def test_sorted_rows_is_the_stable_grouping():
    rng = np.random.default_rng(3)
    idx = rng.integers(0, 13, (31, 4))
    counts, offsets, pair_pos, row_token = sorted_rows(idx, 13, has_shared=True, align=8)
    assert counts[:13].sum() == idx.size and counts[13] == 31
    assert np.all(offsets % 8 == 0)
    flat = idx.reshape(-1)
    for e in range(13):
        rows = pair_pos[flat == e]
        assert np.all(np.diff(rows) == 1) and (rows.size == 0 or rows[0] == offsets[e])
    np.testing.assert_array_equal(row_token[pair_pos], np.arange(idx.size) // 4)
    np.testing.assert_array_equal(row_token[offsets[13]:offsets[13] + 31], np.arange(31))
