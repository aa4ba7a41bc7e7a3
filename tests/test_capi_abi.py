"""The C-ABI library loads and exports every entry point the header declares (no GPU calls)."""
import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def declared_entry_points():
    names = []
    for header in sorted((ROOT / "include").glob("*.h")):
        text = header.read_text()
        names += re.findall(r"WM_EXPORT\s+[\w\s\*]+?\b(wm_\w+)\s*\(", text)
    return names


@pytest.fixture(scope="module")
def library():
    from whallm_b200 import build, lib
    if not lib.LIB_PATH.exists():
        build.build()
    return ctypes.CDLL(str(lib.LIB_PATH))


def test_header_declares_the_binding_list():
    from whallm_b200 import lib
    assert set(declared_entry_points()) == set(lib.EXPORTS)


def test_library_exports_every_declared_symbol(library):
    for name in declared_entry_points():
        assert hasattr(library, name), name


def test_create_fails_cleanly_without_a_b200():
    import torch
    from whallm_b200 import lib
    if torch.cuda.is_available():
        pytest.skip("a GPU is present: the GPU tests cover wm_create")
    with pytest.raises(lib.WMError):
        lib.Context(0, max_tokens=4, max_hidden=64, max_inter=64, max_experts=2, max_topk=1)


def test_binding_struct_layout_matches_header():
    """ctypes structure sizes equal the C compiler's for the header's structs."""
    import subprocess, tempfile
    from whallm_b200 import lib
    src = '#include <stdio.h>\n#include "whallm_moe.h"\nint main(){printf("%zu %zu %zu %zu\\n", sizeof(wm_options), sizeof(wm_matrix), sizeof(wm_moe_args), sizeof(wm_counters));return 0;}\n'
    with tempfile.TemporaryDirectory() as d:
        c = Path(d) / "s.c"
        c.write_text(src)
        exe = Path(d) / "s"
        subprocess.run(["gcc", "-I", str(ROOT / "include"), str(c), "-o", str(exe)], check=True)
        sizes = [int(v) for v in subprocess.run([str(exe)], capture_output=True, text=True).stdout.split()]
    assert sizes == [ctypes.sizeof(lib.Options), ctypes.sizeof(lib.Matrix), ctypes.sizeof(lib.MoeArgs),
                     ctypes.sizeof(lib.Counters)]


def test_binding_flags_match_header():
    """Every WM_FLAG_* of the header has its lib.FLAG_* twin with the same bit, and no other."""
    from whallm_b200 import lib
    text = "".join(h.read_text() for h in sorted((ROOT / "include").glob("*.h")))
    header = {name: int(value) for name, value in re.findall(r"#define\s+WM_(FLAG_\w+)\s+(\d+)", text)}
    binding = {name: getattr(lib, name) for name in dir(lib) if name.startswith("FLAG_")}
    assert header == binding
    bits = list(header.values())
    assert all(b & (b - 1) == 0 for b in bits) and len(set(bits)) == len(bits)
