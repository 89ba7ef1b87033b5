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


def test_no_gpu_fails_loudly(tmp_path):
    """Where there is no GPU, the backend and the host side refuse with an error and a message - no CPU fallback:
    gcuda_open returns NULL with the CUDA error, ghost_open GHOST_E_BACKEND (7) with it and no model."""
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is here")
    from geode_b200 import synth
    L = C.CDLL(LIBS["geode_cuda.h"])
    L.gcuda_open.restype = C.c_void_p
    L.gcuda_open.argtypes = [C.c_int, C.c_char_p, C.c_int]
    err = C.create_string_buffer(512)
    assert not L.gcuda_open(0, err, 512)
    assert err.value
    H = C.CDLL(LIBS["geode_host.h"])
    H.ghost_open.argtypes = [C.c_char_p, C.c_int32, C.c_int32, C.c_int32, C.POINTER(C.c_void_p), C.c_char_p,
                             C.c_size_t]
    d = str(tmp_path / "pack")
    synth.write_pack(d, synth.tiny_shape("qwen35moe", n_layers=2, ctx=64), seed=1)
    m = C.c_void_p(1)
    err = C.create_string_buffer(512)
    assert H.ghost_open(d.encode(), 0, 64, 5, C.byref(m), err, 512) == 7
    assert not m.value and b"gcuda_open" in err.value
