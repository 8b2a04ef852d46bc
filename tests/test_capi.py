"""The C-ABI libraries load and export every function include/*.h declares.
No compute calls: this runs without a GPU."""
import ctypes
import re
from pathlib import Path

import zest_b200 as Z

ROOT = Path(__file__).resolve().parents[1]


def declared(header: str) -> list[str]:
    text = (ROOT / "include" / header).read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(zest_[a-z0-9_]+)\s*\(", text)))


def test_zest_library_exports_header():
    L = ctypes.CDLL(str(Z.LIB_PATH))
    names = declared("zest_b200.h")
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing
    assert sorted(Z.exported_symbols()) == names


def test_version_and_error_without_gpu():
    L = Z.lib()
    assert L.zest_version() == 1
    assert isinstance(L.zest_last_error(), bytes)


def test_header_layout_of_wkey():
    # zest_wkey mirrors xdna_npu::wkey: two pointers, an int, two int64
    assert ctypes.sizeof(Z.WKey) == 40
    assert Z.WKey.K.offset == 24 and Z.WKey.N.offset == 32


def test_binding_signatures_follow_the_header():
    # the ctypes binding declares every entry point with the header's
    # number of parameters
    text = re.sub(r"/\*.*?\*/", "", (ROOT / "include" / "zest_b200.h").read_text(), flags=re.S)
    L = Z.lib()
    checked = 0
    for m in re.finditer(r"\b(zest_[a-z0-9_]+)\s*\(([^;{]*?)\)\s*;", text):
        name, params = m.group(1), m.group(2).strip()
        n = 0 if params in ("", "void") else params.count(",") + 1
        f = getattr(L, name)
        assert f.argtypes is not None, f"{name} has no ctypes signature"
        assert len(f.argtypes) == n, f"{name}: header {n} parameters, binding {len(f.argtypes)}"
        checked += 1
    assert checked >= 30
