"""Blob-layout mirror (expert_layout.py:8-166) on the host (no GPU)."""
import pytest
import torch

from whallm_b200 import layout as L


def test_qwen_blob_size_matches_config_shapes():
    regs = L.qwen_regions(2048, 512)
    assert L.blob_size(regs, L.QWEN_BATCHED) == 1_671_168


def test_fused_blob_size_and_w13_view():
    regs = L.fused_regions(7168, 2048)
    assert L.blob_size(regs, L.FUSED_BATCHED) == 23_396_352
    assert regs["w13.weight"].offset == 0 and regs["w13.weight"].length == 2 * regs["w1.weight"].length
    assert regs["w13.scale"].offset == regs["w3.scale"].offset


def test_fp8_blob_size():
    regs = L.fp8_regions(7168, 2048)
    assert L.blob_size(regs, L.FP8_BATCHED) == 44_050_944


def test_batched_layer_layout_places_regions():
    regs = L.fused_regions(256, 128)
    size = L.blob_size(regs, L.FUSED_BATCHED)
    lay = L.batched_layer_layout(regs, L.FUSED_BATCHED, size, 5)
    base, stride, inner = lay["w1.weight"]
    assert base == 0 and stride == regs["w13.weight"].length and inner == regs["w3.weight"].length
    b2, s2, i2 = lay["w2.scale"]
    assert s2 == regs["w2.scale"].length and i2 == 0
    assert lay["w13.scale"][0] == 5 * (regs["w13.weight"].length + regs["w2.weight"].length)


def test_batched_layer_layout_rejects_bad_partitions():
    regs = L.qwen_regions(256, 128)
    with pytest.raises(ValueError):
        L.batched_layer_layout(regs, ("gate_up.weight", "down.weight"), 0, 2)
    with pytest.raises(ValueError):
        L.batched_layer_layout(regs, L.QWEN_BATCHED, 1, 2)


def test_projection_strides_follow_region_major_views():
    buf = torch.zeros(10 * 96, dtype=torch.uint8)
    w = torch.as_strided(buf, (10, 4, 16), (96, 16, 1), 8)  # expert stride 96, inner offset 8
    s = torch.zeros(10, 4, 2, dtype=torch.uint8)
    p = L.Projection.stacked(w, s)
    assert p.weight_stride == 96 and p.scale_stride == 8


# ---------------------------------------------------------------- pinned by the reference's own layout code
import json
from pathlib import Path

GOLDEN = json.loads((Path(__file__).resolve().parent / "golden" / "expert_layout.json").read_text())


def _regions(table: dict) -> dict:
    return {n: L.Region(n, "U8", (1,), off, ln) for n, (off, ln) in table.items()}


@pytest.mark.parametrize("fmt", GOLDEN["formats"], ids=[f["name"] for f in GOLDEN["formats"]])
def test_slot_regions_match_reference(fmt):
    """qwen_regions / fused_regions give the reference's slot regions (expert_layout.py:8-80)."""
    mine = (L.fused_regions if fmt["kind"] == "fused" else L.qwen_regions)(fmt["hidden"], fmt["inter"])
    assert {n: [r.offset, r.length] for n, r in mine.items()} == fmt["regions"]
    batched = L.FUSED_BATCHED if fmt["kind"] == "fused" else L.QWEN_BATCHED
    assert list(batched) == fmt["batched"]
    assert L.blob_size(mine, batched) == fmt["blob_size"]


@pytest.mark.parametrize("fmt", GOLDEN["formats"], ids=[f["name"] for f in GOLDEN["formats"]])
def test_batched_layer_layout_matches_reference(fmt):
    """batched_layer_layout places every region where expert_layout.py:83-119 does."""
    regs = _regions(fmt["regions"])
    for experts, want in fmt["placements"].items():
        got = L.batched_layer_layout(regs, tuple(fmt["batched"]), fmt["blob_size"], int(experts))
        assert {n: list(v) for n, v in got.items()} == want


def test_batched_layer_layout_refuses_what_reference_refuses():
    for case in GOLDEN["refused"]:
        regs = _regions(case["regions"])
        if case["refused"]:
            with pytest.raises(ValueError):
                L.batched_layer_layout(regs, tuple(case["batched"]), case["blob_size"], 2)
        else:
            L.batched_layer_layout(regs, tuple(case["batched"]), case["blob_size"], 2)
    nested = GOLDEN["nested"]
    got = L.batched_layer_layout(_regions(nested["regions"]), tuple(nested["batched"]), nested["blob_size"],
                                 nested["experts"])
    assert {n: list(v) for n, v in got.items()} == nested["placements"]
