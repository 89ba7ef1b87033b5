"""The C ABI (no GPU needed): every function include/*.h declares is exported by the library that implements it, and
the package fails loudly, instead of falling back, when a library is missing."""
import ctypes as C
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INCLUDE = os.path.join(ROOT, "include")
# header -> the library exporting its functions
LIBS = {
    "geode_cuda.h": os.path.join(ROOT, "geode_b200", "libgeode_cuda.so"),
    "geode_host.h": os.path.join(ROOT, "geode_b200", "libgeode_host.so"),
}


def declared(header: str):
    """Function names declared in a C header (prototypes ending in ');' at file scope, comments removed)."""
    text = open(os.path.join(INCLUDE, header)).read()
    text = re.sub(r"/\*.*?\*/", " ", text, flags=re.S)
    text = re.sub(r"//[^\n]*", " ", text)
    names = re.findall(r"\b([a-z][a-z0-9_]*)\s*\([^;{}]*\)\s*;", text)
    return sorted({n for n in names if not n.startswith(("sizeof", "typedef"))})


@pytest.mark.parametrize("header", sorted(h for h in os.listdir(INCLUDE) if h.endswith(".h")))
def test_header_symbols_exported(header):
    assert header in LIBS, f"{header}: no library recorded for it"
    lib_path = LIBS[header]
    if not os.path.exists(lib_path):
        pytest.fail(f"{lib_path} is not built (python -m geode_b200.build)")
    lib = C.CDLL(lib_path)
    names = declared(header)
    assert names, header
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, f"{header}: declared but not exported: {missing}"


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    import geode_b200

    monkeypatch.setattr(geode_b200, "CUDA_SO", str(tmp_path / "absent.so"))
    monkeypatch.setattr(geode_b200, "_cuda", None)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        geode_b200.cuda_lib()
