"""Regenerate the golden fixtures of this directory from the reference checkout.

Run in a container that has the reference project (yanun0323/Whallm) checked
out; pass its root as the first argument.  Nothing on the GPU box runs this:
the JSON files it writes are committed and the tests read only those.

* mxfp4_kat.json -- the known-answer vectors of the reference's MXFP4
  quantiser, read as text from Tests/DeepSeekRepackTests/DeepSeekRepackTests.swift
  (testMXFP4MatchesMLXFixedVector, testMXFP4MatchesMLXBF16Rows,
  testMXFP4ConvertsOfficialFP8Blocks, testMXFP4FP8ConversionMatchesMLXFixedVector).
  The Swift source builds some inputs with expressions; this script evaluates
  the same expressions in Python and stores the resulting bytes.
* expert_waves.json -- outputs of the reference's own pure-numpy scheduler
  runtime/deepseek_v4_ssd/qwen_expert_waves.py (imported by file path, as the
  reference's portable tests do) on seeded routes.
* expert_layout.json -- outputs of the reference's own blob-layout code,
  runtime/deepseek_v4_ssd/expert_layout.py (_fused_slot_regions,
  _qwen_slot_regions, batched_layer_layout), loaded by file path together with
  the manifest.py it imports (json / dataclasses / pathlib only): the slot
  regions of the reference's three expert formats and their region-major
  placements at several expert counts, plus partitions it refuses.
"""
from __future__ import annotations

import importlib.util
import json
import re
import struct
import sys
from pathlib import Path

import numpy as np

OUT = Path(__file__).resolve().parent


def _swift_array(src: str, anchor: str, name: str) -> list[int]:
    """The integer literals of `let <name>: [...] = [ ... ]` after `anchor`."""
    start = src.index(anchor)
    m = re.search(r"let %s: \[[A-Za-z0-9]+\] = \[(.*?)\]" % name, src[start:], re.S)
    return [int(tok, 0) for tok in re.findall(r"0x[0-9a-fA-F]+|\d+", m.group(1))]


def _expected_bytes(src: str, anchor: str) -> list[dict]:
    """Every XCTAssertEqual([UInt8](result....), [...]) byte list after `anchor`."""
    start = src.index(anchor)
    end = src.index("func test", start + len(anchor))
    body = src[start:end]
    out = []
    for m in re.finditer(r"XCTAssertEqual\(\s*\[UInt8\]\(result\.(\w+)[^)]*\)\)?,\s*(.*?)\)\n", body, re.S):
        expr = m.group(2)
        lit = re.search(r"\[(.*?)\]", expr, re.S)
        values = [int(tok, 0) for tok in re.findall(r"0x[0-9a-fA-F]+|\b\d+\b", lit.group(1))]
        rep = re.search(r"Array\(repeating: (\d+), count: (\d+)\)", expr)
        if rep:
            values += [int(rep.group(1))] * int(rep.group(2))
        out.append({"field": m.group(1), "bytes": values})
    return out


def _bf16_bits(v: float) -> int:
    return struct.unpack("<I", struct.pack("<f", v))[0] >> 16


def mxfp4_kat(ref: Path) -> dict:
    src = (ref / "Tests/DeepSeekRepackTests/DeepSeekRepackTests.swift").read_text()
    cases = []

    # testMXFP4MatchesMLXFixedVector: 14 literal floats then 18 zeros, one 1x32 row.
    anchor = "func testMXFP4MatchesMLXFixedVector"
    start = src.index(anchor)
    lit = re.search(r"let values: \[Float\] = \[(.*?)\]", src[start:], re.S).group(1)
    floats = [float(t) for t in re.findall(r"-?\d+(?:\.\d+)?", lit)]
    zeros = int(re.search(r"Array\(repeating: 0, count: (\d+)\)", src[start:]).group(1))
    values = floats + [0.0] * zeros
    cases.append({"name": "MatchesMLXFixedVector", "kind": "bf16", "rows": 1, "cols": 32,
                  "source_bf16": [_bf16_bits(v) for v in values],
                  "expect": _expected_bytes(src, anchor),
                  "ref": "Tests/DeepSeekRepackTests/DeepSeekRepackTests.swift:336-351"})

    # testMXFP4MatchesMLXBF16Rows: 64 literal bf16 bit patterns, two rows.
    anchor = "func testMXFP4MatchesMLXBF16Rows"
    bits = _swift_array(src, anchor, "bits")
    cases.append({"name": "MatchesMLXBF16Rows", "kind": "bf16", "rows": 2, "cols": 32,
                  "source_bf16": bits, "expect": _expected_bytes(src, anchor),
                  "ref": "Tests/DeepSeekRepackTests/DeepSeekRepackTests.swift:353-375"})

    # testMXFP4ConvertsOfficialFP8Blocks: first row literal + zeros, 128x128, inverse scale bytes.
    anchor = "func testMXFP4ConvertsOfficialFP8Blocks"
    first = _swift_array(src, anchor, "firstRow")
    start = src.index(anchor)
    first += [0] * int(re.search(r"Array\(repeating: 0, count: (\d+)\)", src[start:]).group(1))
    inv = [int(t, 16) for t in re.search(r"inverseScales: Data\(\[(.*?)\]\)", src[start:]).group(1).replace("0x", "").split(", ")]
    source = first + [0] * (127 * 128)
    cases.append({"name": "ConvertsOfficialFP8Blocks", "kind": "fp8", "rows": 128, "cols": 128,
                  "source_u8": source, "inverse_scale_bytes": inv,
                  "expect": _expected_bytes(src, anchor),
                  "ref": "Tests/DeepSeekRepackTests/DeepSeekRepackTests.swift:377-393"})

    # testMXFP4FP8ConversionMatchesMLXFixedVector: value = UInt8(truncating: i*37+11), NaN codes
    # avoided by flipping the low bit; checked by SHA-256 of weights and scales.
    anchor = "func testMXFP4FP8ConversionMatchesMLXFixedVector"
    start = src.index(anchor)
    body = src[start:src.index("func test", start + len(anchor))]
    mul, add = (int(v) for v in re.search(r"index \* (\d+) \+ (\d+)", body).groups())
    inv = [int(t, 16) for t in re.search(r"inverseScales: Data\(\[(.*?)\]\)", body).group(1).replace("0x", "").split(", ")]
    source = []
    for i in range(128 * 128):
        v = (i * mul + add) & 0xFF
        source.append(v ^ 1 if v & 0x7F == 0x7F else v)
    shas = re.findall(r'"([0-9a-f]{64})"', body)
    cases.append({"name": "FP8ConversionMatchesMLXFixedVector", "kind": "fp8", "rows": 128, "cols": 128,
                  "source_u8": source, "inverse_scale_bytes": inv,
                  "expect_sha256": {"weights": shas[0], "scales": shas[1]},
                  "ref": "Tests/DeepSeekRepackTests/DeepSeekRepackTests.swift:395-415"})
    return {"generator": "tests/golden/make_golden.py", "cases": cases}


def expert_waves_fixture(ref: Path) -> dict:
    path = ref / "runtime/deepseek_v4_ssd/qwen_expert_waves.py"
    spec = importlib.util.spec_from_file_location("_ref_qwen_expert_waves", path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod
    spec.loader.exec_module(mod)
    rng = np.random.default_rng(20260921)
    cases = []
    for tokens, k, experts in ((1, 10, 512), (17, 10, 512), (128, 8, 64), (9, 10, 512)):
        if tokens == 9:
            selected = np.full((tokens, k), 5, dtype=np.int32)
        else:
            selected = rng.integers(0, experts, size=(tokens, k), dtype=np.int32)
        for capacity in (1, 3, 32, 1024):
            waves = [[[int(e), [int(p) for p in pos]] for e, pos in w.groups]
                     for w in mod.expert_waves(selected, capacity, experts)]
            cases.append({"selected": selected.tolist(), "capacity": capacity, "experts": experts, "waves": waves})
    return {"generator": "tests/golden/make_golden.py",
            "ref": "runtime/deepseek_v4_ssd/qwen_expert_waves.py:23-51", "cases": cases}


def _load_layout_modules(ref: Path):
    """manifest.py and expert_layout.py as one package (expert_layout imports .manifest)."""
    import types
    pkg_dir = ref / "runtime/deepseek_v4_ssd"
    pkg = types.ModuleType("_ref_ds")
    pkg.__path__ = [str(pkg_dir)]
    sys.modules["_ref_ds"] = pkg
    mods = {}
    for name in ("manifest", "expert_layout"):
        spec = importlib.util.spec_from_file_location(f"_ref_ds.{name}", pkg_dir / f"{name}.py")
        mod = importlib.util.module_from_spec(spec)
        sys.modules[spec.name] = mod
        spec.loader.exec_module(mod)
        mods[name] = mod
    return mods["manifest"], mods["expert_layout"]


def expert_layout_fixture(ref: Path) -> dict:
    manifest, layout = _load_layout_modules(ref)
    from types import SimpleNamespace

    def regions_json(regs):
        return {n: [r.offset, r.length] for n, r in regs.items()}

    formats = []
    for label, table, kind in (("deepseek", manifest.EXPERT_REGIONS, "fused"),
                               ("deepseek_v41", manifest.DEEPSEEK_V41_EXPERT_REGIONS, "fused"),
                               ("qwen", manifest.QWEN_EXPERT_REGIONS, "qwen")):
        tensors = tuple(manifest.Tensor(n, d, tuple(sh), off, ln) for n, d, sh, off, ln in table)
        model = SimpleNamespace(expert_regions=tensors, expert_blob_size=sum(t.length for t in tensors))
        if kind == "fused":
            regs = layout._fused_slot_regions(model)
            batched = layout.FusedMXFP4Layout.batched_regions
        else:
            regs = layout._qwen_slot_regions(model)
            batched = layout.GateUpMXFP4Layout.batched_regions
        w1 = {n: sh for n, _, sh, _, _ in table}
        if kind == "fused":
            inter, hidden = w1["w1.weight"][0], 2 * w1["w1.weight"][1]
        else:
            inter, hidden = w1["gate_up.weight"][0] // 2, 8 * w1["gate_up.weight"][1]
        placements = {}
        for experts in (1, 3, 384):
            got = layout.batched_layer_layout(regs, batched, model.expert_blob_size, experts)
            placements[str(experts)] = {n: list(v) for n, v in got.items()}
        formats.append({"name": label, "kind": kind, "hidden": hidden, "inter": inter,
                        "blob_size": model.expert_blob_size, "batched": list(batched),
                        "regions": regions_json(regs), "placements": placements})

    # partitions the reference refuses (gap, short cover, region outside every batched region)
    tensors = {n: manifest.Tensor(n, "U8", (1,), off, ln) for n, off, ln in
               (("a", 0, 16), ("b", 16, 8), ("c", 24, 40), ("inner", 20, 4), ("straddle", 12, 8))}
    refused = []
    for names, batched, blob in ((("a", "c"), ("a", "c"), 64), (("a", "b", "c"), ("a", "b", "c"), 65),
                                 (("a", "b", "c", "straddle"), ("a", "b", "c"), 64)):
        regs = {n: tensors[n] for n in names}
        try:
            layout.batched_layer_layout(regs, batched, blob, 2)
            refused.append({"regions": regions_json(regs), "batched": list(batched), "blob_size": blob,
                            "refused": False})
        except ValueError:
            refused.append({"regions": regions_json(regs), "batched": list(batched), "blob_size": blob,
                            "refused": True})
    regs = {n: tensors[n] for n in ("a", "b", "c", "inner")}
    accepted = {n: list(v) for n, v in layout.batched_layer_layout(regs, ("a", "b", "c"), 64, 5).items()}
    return {"generator": "tests/golden/make_golden.py",
            "ref": "runtime/deepseek_v4_ssd/expert_layout.py:8-119, manifest.py:17-45",
            "formats": formats, "refused": refused,
            "nested": {"regions": regions_json(regs), "batched": ["a", "b", "c"], "blob_size": 64, "experts": 5,
                       "placements": accepted}}


def main() -> None:
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_golden.py <reference checkout root>")
    ref = Path(sys.argv[1])
    kat = mxfp4_kat(ref)
    (OUT / "mxfp4_kat.json").write_text(json.dumps(kat, separators=(",", ":")) + "\n")
    waves = expert_waves_fixture(ref)
    (OUT / "expert_waves.json").write_text(json.dumps(waves, separators=(",", ":")) + "\n")
    lay = expert_layout_fixture(ref)
    (OUT / "expert_layout.json").write_text(json.dumps(lay, separators=(",", ":")) + "\n")
    for case in kat["cases"]:
        print(case["name"], {k: (len(v) if isinstance(v, list) else v) for k, v in case.items() if k != "name"})
    print("waves cases:", len(waves["cases"]))


if __name__ == "__main__":
    main()
