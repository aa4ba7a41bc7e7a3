"""HBM expert store: an installed model's expert layer files, resident in device memory.

The reference keeps experts on SSD and streams slots into a slot cache
(runtime/deepseek_v4_ssd/expert_cache.py:382-420, 2059-2084).  A B200 holds
every layer of these models in HBM, so here a layer file is copied to the
device once and the expert kernels read its bytes in place.

* Manifest checks follow runtime/deepseek_v4_ssd/manifest.py:150-200: unique
  file entries, files inside the model root with the recorded sizes, and
  ``experts/layer_XX.bin`` exactly ``expertCount * expertBlobSize`` bytes
  (manifest.py:171-173); the expert regions must partition one blob
  (expert_layout.py:8-80: the Qwen gate_up/down regions, the fused
  w3 | w1 | w2 | w3.s | w1.s | w2.s slot, and this library's FP8 blob).
* Copy: the file is read in chunks into two pinned host buffers while the
  previous chunk travels to HBM on a side stream (reads overlap copies).
* Views: the slot-major file bytes are used as they are -- expert e of a
  region at ``base + e * blob_size + offset`` -- or, on request, a
  region-major layer buffer placed by ``batched_layer_layout``
  (expert_layout.py:83-119), the layout the reference's batched views use.
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass
from pathlib import Path

import torch

from . import lib
from .layout import FP8_BATCHED, FUSED_BATCHED, QWEN_BATCHED, Projection, Region, batched_layer_layout
from .moe import LayerWeights

QWEN_REGION_NAMES = frozenset({"gate_up.weight", "gate_up.scale", "down.weight", "down.scale"})
FUSED_REGION_NAMES = frozenset({"w1.weight", "w1.scale", "w2.weight", "w2.scale", "w3.weight", "w3.scale"})
FP8_REGION_NAMES = frozenset({"w13.weight", "w2.weight", "w13.scale", "w2.scale"})


def layer_path(layer: int) -> str:
    """Relative path of a layer's expert file (manifest.py:172-173)."""
    return f"experts/layer_{layer:02d}.bin"


@dataclass(frozen=True)
class ExpertManifest:
    """The expert part of an installed model's manifest.json."""
    root: Path
    layer_count: int
    expert_count: int
    selected_expert_count: int
    expert_blob_size: int
    regions: dict[str, Region]   # slot regions; the fused layout adds w13.weight / w13.scale
    layout: int                  # lib.LAYOUT_*
    H: int
    I: int
    files: dict[str, int]

    @property
    def batched(self) -> tuple[str, ...]:
        return {lib.LAYOUT_QWEN_GATE_UP_MXFP4: QWEN_BATCHED, lib.LAYOUT_DS_W13_MXFP4: FUSED_BATCHED,
                lib.LAYOUT_W13_FP8_B128: FP8_BATCHED}[self.layout]


def _regions_of(raw: dict) -> dict[str, Region]:
    out: dict[str, Region] = {}
    for item in raw.get("expertRegions", []):
        r = Region(item["name"], item["dtype"], tuple(item["shape"]), int(item["offset"]), int(item["length"]))
        if r.name in out:
            raise ValueError(f"expert region {r.name} appears twice")
        out[r.name] = r
    return out


def _check_partition(regions: dict[str, Region], names, blob: int) -> None:
    spans = sorted((regions[n].offset, regions[n].length, n) for n in names)
    expected = 0
    for offset, length, name in spans:
        if offset != expected or length <= 0:
            raise ValueError(f"expert region {name} does not partition the blob")
        expected += length
    if expected != blob:
        raise ValueError("expert regions do not cover the expert blob")


def _fused_slot(regions: dict[str, Region], blob: int) -> dict[str, Region]:
    """The fused slot (expert_layout.py:8-63): w3 | w1 | w2 | w3.s | w1.s | w2.s
    with the virtual w13 = [w3; w1]; the blob's own offsets must be these."""
    w1, w3, s1, s3 = regions["w1.weight"], regions["w3.weight"], regions["w1.scale"], regions["w3.scale"]
    if w1.dtype != w3.dtype or w1.shape[1:] != w3.shape[1:]:
        raise ValueError(f"w1 ({w1.dtype}, {w1.shape}) and w3 ({w3.dtype}, {w3.shape}) differ in type or row shape: no fused w13 view")
    if s1.dtype != s3.dtype or s1.shape[1:] != s3.shape[1:]:
        raise ValueError(f"w1.scale ({s1.dtype}, {s1.shape}) and w3.scale ({s3.dtype}, {s3.shape}) differ in type or row shape: no fused w13 view")
    slot, off = {}, 0
    for name in ("w3.weight", "w1.weight", "w2.weight", "w3.scale", "w1.scale", "w2.scale"):
        src = regions[name]
        if src.offset != off:
            raise ValueError(f"region {name} is not where the fused slot places it")
        slot[name] = src
        off += src.length
    if off != blob:
        raise ValueError(f"the fused slot adds up to {off} bytes, the manifest says {blob}")
    slot["w13.weight"] = Region("w13.weight", w3.dtype, (w3.shape[0] + w1.shape[0], *w3.shape[1:]), 0,
                                w3.length + w1.length)
    slot["w13.scale"] = Region("w13.scale", s3.dtype, (s3.shape[0] + s1.shape[0], *s3.shape[1:]), s3.offset,
                               s3.length + s1.length)
    return slot


def read_manifest(root: str | os.PathLike) -> ExpertManifest:
    """Parse and check the expert part of ``root/manifest.json`` (manifest.py:150-200)."""
    root = Path(root).resolve()
    with (root / "manifest.json").open("rb") as f:
        raw = json.load(f)
    files = {item["path"]: int(item["size"]) for item in raw.get("files", [])}
    if len(files) != len(raw.get("files", [])):
        raise ValueError("manifest.json lists a file path more than once")
    for path, size in files.items():
        target = (root / path).resolve()
        if root not in target.parents or not target.is_file():
            raise ValueError(f"manifest file {path} lies outside the model directory or does not exist")
        if target.stat().st_size != size:
            raise ValueError(f"{path} has {target.stat().st_size} bytes, manifest.json says {size}")
    try:
        layers, experts = int(raw["layerCount"]), int(raw["expertCount"])
        selected, blob = int(raw["selectedExpertCount"]), int(raw["expertBlobSize"])
    except KeyError as exc:
        raise ValueError(f"manifest lacks {exc.args[0]}") from None
    if layers <= 0 or experts <= 0 or blob <= 0 or not 0 < selected <= experts:
        raise ValueError("manifest expert counts are not positive")
    for layer in range(layers):
        path = layer_path(layer)
        if path not in files:
            raise ValueError(f"manifest.json lists no {path}")
        if files[path] != experts * blob:
            raise ValueError(f"{path} has {files[path]} bytes, expected {experts} experts x {blob} bytes")
    regions = _regions_of(raw)
    names = frozenset(regions)
    if names == QWEN_REGION_NAMES:
        _check_partition(regions, QWEN_REGION_NAMES, blob)
        gu, dn = regions["gate_up.weight"], regions["down.weight"]
        I, H = gu.shape[0] // 2, gu.shape[1] * 8
        layout = lib.LAYOUT_QWEN_GATE_UP_MXFP4
        ok = (gu.dtype == "U32" and tuple(dn.shape) == (H, I // 8) and gu.length == 2 * I * H // 2
              and regions["gate_up.scale"].length == 2 * I * H // 32 and regions["down.scale"].length == H * I // 32)
    elif names == FUSED_REGION_NAMES:
        regions = _fused_slot(regions, blob)
        w1, w2 = regions["w1.weight"], regions["w2.weight"]
        I, H = w1.shape[0], w1.shape[1] * 8
        layout = lib.LAYOUT_DS_W13_MXFP4
        ok = (w1.dtype == "U32" and tuple(w2.shape) == (H, I // 8) and w1.length == I * H // 2
              and regions["w13.scale"].length == 2 * I * H // 32 and regions["w2.scale"].length == H * I // 32)
    elif names == FP8_REGION_NAMES:
        _check_partition(regions, FP8_REGION_NAMES, blob)
        w13, w2 = regions["w13.weight"], regions["w2.weight"]
        I, H = w13.shape[0] // 2, w13.shape[1]
        layout = lib.LAYOUT_W13_FP8_B128
        ok = (w13.dtype == "F8_E4M3" and tuple(w2.shape) == (H, I) and w13.length == 2 * I * H
              and regions["w13.scale"].length == 4 * (2 * I // 128) * (H // 128)
              and regions["w2.scale"].length == 4 * (H // 128) * (I // 128))
    else:
        raise ValueError(f"unknown expert blob regions {sorted(names)}")
    if not ok:
        raise ValueError("expert region shapes or sizes are inconsistent")
    return ExpertManifest(root, layers, experts, selected, blob, regions, layout, H, I, files)


def write_manifest(root: str | os.PathLike, layer_count: int, expert_count: int, selected_expert_count: int,
                   regions: dict[str, Region], extra: dict | None = None) -> Path:
    """Write ``manifest.json`` for expert layer files already under ``root``
    (the fields read_manifest checks; for tests and synthetic installs)."""
    root = Path(root)
    blob = max(r.offset + r.length for r in regions.values())
    files = [{"path": layer_path(i), "size": (root / layer_path(i)).stat().st_size} for i in range(layer_count)]
    raw = {"layerCount": layer_count, "expertCount": expert_count, "selectedExpertCount": selected_expert_count,
           "expertBlobSize": blob, "files": files,
           "expertRegions": [{"name": r.name, "dtype": r.dtype, "shape": list(r.shape), "offset": r.offset,
                              "length": r.length} for r in regions.values()]}
    raw.update(extra or {})
    path = root / "manifest.json"
    path.write_text(json.dumps(raw, indent=1))
    return path


def slot_regions(layout: int, H: int, I: int) -> dict[str, Region]:
    """The blob regions this library writes for a layout (reference orders)."""
    from .layout import fp8_regions, fused_regions, qwen_regions
    if layout == lib.LAYOUT_QWEN_GATE_UP_MXFP4:
        return qwen_regions(H, I)
    if layout == lib.LAYOUT_DS_W13_MXFP4:
        regs = fused_regions(H, I)
        return {n: r for n, r in regs.items() if n not in ("w13.weight", "w13.scale")}
    if layout == lib.LAYOUT_W13_FP8_B128:
        return fp8_regions(H, I)
    raise ValueError(f"unknown layout {layout}")


def pack_layer(layout: int, H: int, I: int, w13: torch.Tensor, s13: torch.Tensor, w2: torch.Tensor,
               s2: torch.Tensor) -> torch.Tensor:
    """Slot-major layer bytes [E, blob] from per-expert projections ([E, rows, row bytes] uint8 weights and
    scales; fp32 scales for FP8); the fused layout splits w13 = [w3; w1]."""
    regs = slot_regions(layout, H, I)
    E = w13.shape[0]
    blob = max(r.offset + r.length for r in regs.values())
    out = torch.empty((E, blob), dtype=torch.uint8, device=w13.device)

    def put(name: str, t: torch.Tensor) -> None:
        r = regs[name]
        b = t.reshape(E, -1).contiguous().view(torch.uint8)
        if b.shape[1] != r.length:
            raise ValueError(f"{name}: {b.shape[1]} bytes per expert, region holds {r.length}")
        out[:, r.offset:r.offset + r.length] = b

    if layout == lib.LAYOUT_QWEN_GATE_UP_MXFP4:
        put("gate_up.weight", w13), put("gate_up.scale", s13), put("down.weight", w2), put("down.scale", s2)
    elif layout == lib.LAYOUT_DS_W13_MXFP4:
        put("w3.weight", w13[:, :I]), put("w1.weight", w13[:, I:]), put("w2.weight", w2)
        put("w3.scale", s13[:, :I]), put("w1.scale", s13[:, I:]), put("w2.scale", s2)
    else:
        put("w13.weight", w13), put("w2.weight", w2), put("w13.scale", s13), put("w2.scale", s2)
    return out


@dataclass
class StoreLayer:
    """One layer resident in device memory: its bytes and the expert projections over them."""
    data: torch.Tensor           # uint8: slot-major [E * blob] or region-major layer buffer
    layout: int
    H: int
    I: int
    E: int
    w13: Projection
    w2: Projection
    region_major: bool

    def layer_weights(self, **kw) -> LayerWeights:
        """LayerWeights over these bytes (add the shared expert and router from the common tensors)."""
        return LayerWeights(self.layout, self.H, self.I, self.E, self.w13, self.w2, keep=[self.data], **kw)


def _read_file_into(path: Path, dst: torch.Tensor, chunk_bytes: int) -> None:
    """The whole file into the uint8 tensor `dst`; on a GPU through two pinned
    host buffers, the next chunk's read overlapping the previous chunk's copy."""
    n = dst.numel()
    if Path(path).stat().st_size != n:
        raise ValueError(f"{path} holds {Path(path).stat().st_size} bytes, expected {n}")

    def fill(f, view: memoryview) -> None:
        got = 0
        while got < len(view):
            k = f.readinto(view[got:])
            if not k:
                raise ValueError(f"{path} ended early")
            got += k

    with open(path, "rb", buffering=0) as f:
        if dst.device.type != "cuda":
            fill(f, memoryview(dst.numpy()))
            return
        chunk_bytes = max(1 << 20, min(chunk_bytes, n))
        stream = torch.cuda.Stream(device=dst.device)
        bufs = [torch.empty(chunk_bytes, dtype=torch.uint8, pin_memory=True) for _ in range(2)]
        done: list[torch.cuda.Event | None] = [None, None]
        off, i = 0, 0
        while off < n:
            k = min(chunk_bytes, n - off)
            slot = i & 1
            if done[slot] is not None:
                done[slot].synchronize()  # the buffer's previous copy has left it
            fill(f, memoryview(bufs[slot].numpy())[:k])
            with torch.cuda.stream(stream):
                dst[off:off + k].copy_(bufs[slot][:k], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(stream)
            done[slot] = ev
            off += k
            i += 1
        torch.cuda.current_stream(dst.device).wait_stream(stream)
        stream.synchronize()  # the pinned buffers are released on return


def _strided(buf: torch.Tensor, E: int, stride: int, offset: int, shape: tuple[int, ...],
             dtype: torch.dtype) -> torch.Tensor:
    """[E, *shape] view of `dtype` elements: expert e at byte offset + e * stride of `buf`."""
    es = torch.empty((), dtype=dtype).element_size()
    if offset % es or stride % es:
        raise ValueError("region is not aligned to its element size")
    typed = buf.view(dtype)
    inner = [1]
    for d in reversed(shape[1:]):
        inner.insert(0, inner[0] * d)
    return typed.as_strided((E, *shape), (stride // es, *inner), typed.storage_offset() + offset // es)


class ExpertStore:
    """The expert layer files of an installed model, loaded into device memory."""

    def __init__(self, root: str | os.PathLike):
        self.manifest = read_manifest(root)

    def _projections(self, data: torch.Tensor, places: dict[str, tuple[int, int, int]]):
        m = self.manifest
        H, I, E = m.H, m.I, m.expert_count
        if m.layout == lib.LAYOUT_QWEN_GATE_UP_MXFP4:
            names = ("gate_up.weight", "gate_up.scale", "down.weight", "down.scale")
        else:
            names = ("w13.weight", "w13.scale", "w2.weight", "w2.scale")
        if m.layout == lib.LAYOUT_W13_FP8_B128:
            shapes = ((2 * I, H), (2 * I // 128, H // 128), (H, I), (H // 128, I // 128))
            dtypes = (torch.uint8, torch.float32, torch.uint8, torch.float32)
        else:
            shapes = ((2 * I, H // 2), (2 * I, H // 32), (H, I // 2), (H, I // 32))
            dtypes = (torch.uint8,) * 4
        views = []
        for name, shape, dt in zip(names, shapes, dtypes):
            base, stride, inner = places[name]
            views.append(_strided(data, E, stride, base + inner, shape, dt))
        return Projection.stacked(views[0], views[1]), Projection.stacked(views[2], views[3])

    def load_layer(self, layer: int, device="cuda", region_major: bool = False,
                   chunk_bytes: int = 64 << 20) -> StoreLayer:
        """Layer `layer`'s experts in device memory.  Slot-major (the file's
        bytes as they are) unless `region_major`, which regroups them into the
        batched layer buffer of batched_layer_layout."""
        m = self.manifest
        if not 0 <= layer < m.layer_count:
            raise ValueError(f"layer {layer} outside [0, {m.layer_count})")
        E, blob = m.expert_count, m.expert_blob_size
        data = torch.empty(E * blob, dtype=torch.uint8, device=torch.device(device))
        _read_file_into(m.root / layer_path(layer), data, chunk_bytes)
        if region_major:
            places = batched_layer_layout(m.regions, m.batched, blob, E)
            packed = torch.empty_like(data)
            slots = data.view(E, blob)
            for name in m.batched:
                r = m.regions[name]
                base = places[name][0]
                packed[base:base + E * r.length].view(E, r.length).copy_(slots[:, r.offset:r.offset + r.length])
            data = packed
        else:
            places = {name: (0, blob, r.offset) for name, r in m.regions.items()}
        w13, w2 = self._projections(data, places)
        return StoreLayer(data, m.layout, m.H, m.I, E, w13, w2, region_major)
