"""HBM expert store: manifest checks, slot packing and the views over loaded
layer files (CPU), and layers loaded onto the GPU against in-memory weights.

The manifest fields and checks mirror runtime/deepseek_v4_ssd/manifest.py:150-200
and expert_layout.py:8-166; every file here is synthetic (seeded)."""
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from whallm_b200 import lib, synth
from whallm_b200.store import ExpertStore, layer_path, pack_layer, read_manifest, slot_regions, write_manifest

LAYOUTS = [lib.LAYOUT_QWEN_GATE_UP_MXFP4, lib.LAYOUT_DS_W13_MXFP4, lib.LAYOUT_W13_FP8_B128]


def _weights(layout, E, H, I, seed):
    g = torch.Generator().manual_seed(seed)
    proj = synth.fp8_projection if layout == lib.LAYOUT_W13_FP8_B128 else synth.mxfp4_projection
    w13, s13 = proj(E, 2 * I, H, g, "cpu")
    w2, s2 = proj(E, H, I, g, "cpu")
    return w13, s13, w2, s2


def _install(root: Path, layout, E, H, I, layers=2, seed=0):
    (root / "experts").mkdir(parents=True, exist_ok=True)
    ws = []
    for layer in range(layers):
        w = _weights(layout, E, H, I, seed + layer)
        pack_layer(layout, H, I, *w).numpy().tofile(root / layer_path(layer))
        ws.append(w)
    write_manifest(root, layers, E, 2, slot_regions(layout, H, I))
    return ws


@pytest.mark.parametrize("layout", LAYOUTS)
@pytest.mark.parametrize("region_major", [False, True])
def test_loaded_views_hold_the_packed_weights(tmp_path, layout, region_major):
    E, H, I = 4, 256, 128
    ws = _install(tmp_path, layout, E, H, I)
    m = read_manifest(tmp_path)
    assert (m.layout, m.H, m.I, m.expert_count, m.layer_count) == (layout, H, I, E, 2)
    store = ExpertStore(tmp_path)
    for layer in range(2):
        sl = store.load_layer(layer, device="cpu", region_major=region_major)
        w13, s13, w2, s2 = ws[layer]
        assert torch.equal(sl.w13.weight, w13) and torch.equal(sl.w13.scale, s13)
        assert torch.equal(sl.w2.weight, w2) and torch.equal(sl.w2.scale, s2)
        # expert strides: the slot size in the file's order, the region size when regrouped
        assert sl.w13.weight_stride == (m.regions[m.batched[0]].length if region_major else m.expert_blob_size)


def test_fused_blob_orders_up_rows_first(tmp_path):
    """w13 = [w3; w1]: the blob holds w3 (up) before w1 (gate), expert_layout.py:43-63."""
    E, H, I = 2, 256, 128
    w13, *_ = _install(tmp_path, lib.LAYOUT_DS_W13_MXFP4, E, H, I, layers=1)[0]
    raw = json.loads((tmp_path / "manifest.json").read_text())
    regs = {r["name"]: r for r in raw["expertRegions"]}
    assert regs["w3.weight"]["offset"] == 0 and regs["w1.weight"]["offset"] == I * H // 2
    blob = np.fromfile(tmp_path / layer_path(0), dtype=np.uint8).reshape(E, -1)
    assert np.array_equal(blob[0, :I * H // 2], w13[0, :I].reshape(-1).numpy())


def _manifest(tmp_path) -> dict:
    return json.loads((tmp_path / "manifest.json").read_text())


def _rewrite(tmp_path, raw) -> None:
    (tmp_path / "manifest.json").write_text(json.dumps(raw))


def test_manifest_rejects_bad_installs(tmp_path):
    _install(tmp_path, lib.LAYOUT_QWEN_GATE_UP_MXFP4, 2, 256, 128)
    good = _manifest(tmp_path)
    read_manifest(tmp_path)

    raw = dict(good, files=good["files"] + [good["files"][0]])
    _rewrite(tmp_path, raw)
    with pytest.raises(ValueError, match="more than once"):
        read_manifest(tmp_path)

    raw = dict(good, files=[dict(good["files"][0], path="../outside.bin")] + good["files"][1:])
    _rewrite(tmp_path, raw)
    with pytest.raises(ValueError, match="outside the model directory or does not exist"):
        read_manifest(tmp_path)

    raw = dict(good, files=[dict(good["files"][0], size=good["files"][0]["size"] + 1)] + good["files"][1:])
    _rewrite(tmp_path, raw)
    with pytest.raises(ValueError, match="manifest.json says"):
        read_manifest(tmp_path)

    raw = dict(good, layerCount=3)
    _rewrite(tmp_path, raw)
    with pytest.raises(ValueError, match="lists no experts/layer_02.bin"):
        read_manifest(tmp_path)

    raw = dict(good, expertCount=3)
    _rewrite(tmp_path, raw)
    with pytest.raises(ValueError, match="experts x"):
        read_manifest(tmp_path)

    regions = [dict(r) for r in good["expertRegions"]]
    regions[1]["offset"] += 16  # a gap between gate_up.weight and gate_up.scale
    _rewrite(tmp_path, dict(good, expertRegions=regions))
    with pytest.raises(ValueError, match="partition"):
        read_manifest(tmp_path)

    regions = [dict(r) for r in good["expertRegions"]]
    regions[0]["name"] = "gate.weight"
    _rewrite(tmp_path, dict(good, expertRegions=regions))
    with pytest.raises(ValueError, match="unknown expert blob regions"):
        read_manifest(tmp_path)

    _rewrite(tmp_path, good)
    with pytest.raises(ValueError, match="outside"):
        ExpertStore(tmp_path).load_layer(2, device="cpu")


def test_fused_regions_must_sit_in_slot_order(tmp_path):
    _install(tmp_path, lib.LAYOUT_DS_W13_MXFP4, 2, 256, 128, layers=1)
    raw = _manifest(tmp_path)
    regs = {r["name"]: r for r in raw["expertRegions"]}
    regs["w3.weight"]["offset"], regs["w1.weight"]["offset"] = regs["w1.weight"]["offset"], 0
    _rewrite(tmp_path, dict(raw, expertRegions=list(regs.values())))
    with pytest.raises(ValueError, match="fused slot"):
        read_manifest(tmp_path)


@pytest.mark.gpu
@pytest.mark.parametrize("layout", LAYOUTS)
@pytest.mark.parametrize("region_major", [False, True])
def test_gpu_layer_from_files_equals_in_memory_layer(tmp_path, layout, region_major):
    """The same bytes through the file store and through stacked tensors give
    the same expert rows, bit for bit (the kernels read the bytes in place)."""
    from whallm_b200.layout import Projection
    from whallm_b200.moe import Engine, LayerWeights
    E, H, I, T, K = 16, 1024, 512, 24, 4
    w13, s13, w2, s2 = _install(tmp_path, layout, E, H, I, layers=1, seed=7)[0]
    store = ExpertStore(tmp_path).load_layer(0, device="cuda", region_major=region_major, chunk_bytes=1 << 20)
    dev = "cuda"
    ref = LayerWeights(layout, H, I, E, Projection.stacked(w13.to(dev), s13.to(dev)),
                       Projection.stacked(w2.to(dev), s2.to(dev)))
    eng = Engine(0, max_tokens=64, hidden=H, inter=I, experts=E, topk=K)
    g = torch.Generator(device=dev).manual_seed(3)
    x = synth.activations(T, H, g, dev)
    idx = torch.stack([torch.randperm(E, generator=g, device=dev)[:K] for _ in range(T)]).to(torch.int32)
    a = eng.expert_pairs(store.layer_weights(), x, idx)
    b = eng.expert_pairs(ref, x, idx)
    eng.sync()
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))
    eng.ctx.close()
