"""The tcgen05 descriptors the kernels build by hand (geode_b200/csrc/umma.cuh: the shared-memory matrix descriptor of
the K-major no-swizzle layout and the int8 MMA's instruction descriptor) equal CuTe's own builders (make_umma_desc,
make_instr_desc) for the same operand layouts and shapes - a host-only check (nvcc compiles tests/native/
umma_desc_check.cu against the CUTLASS headers the image vendors; skipped where they or nvcc are absent)."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _cutlass_include():
    try:
        import flashinfer
        p = os.path.join(os.path.dirname(flashinfer.__file__), "data", "cutlass", "include")
        return p if os.path.isdir(os.path.join(p, "cute")) else None
    except Exception:
        return None


def test_umma_descriptors_match_cute(tmp_path):
    inc = _cutlass_include()
    nvcc = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
    if not inc or not (os.path.exists(nvcc) or shutil.which("nvcc")):
        pytest.skip("CUTLASS headers or nvcc not here")
    exe = str(tmp_path / "umma_check")
    subprocess.check_call([nvcc, "-std=c++17", "-I" + inc, "-x", "cu", "-o", exe,
                           os.path.join(ROOT, "tests", "native", "umma_desc_check.cu")],
                          stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
    out = subprocess.run([exe], capture_output=True, text=True)
    assert out.returncode == 0, out.stdout
