"""The device's float exp (expf_ref, geode_b200/csrc/common.cuh) against this host's glibc expf - the reference's float
exp (std::exp on a float) - on all 2^32 floats, through the test hook gcuda_debug_expf_table: the device tabulates
2^28 inputs at a time, the oracle's go_expf_check_table compares them with glibc bit for bit (two NaNs count as
equal). Router weights, silu / sigmoid gates and sampled acceptance rest on this."""
import ctypes as C
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")

import oracle_py as op  # noqa: E402

pytestmark = pytest.mark.gpu


def test_device_expf_equals_glibc_on_every_float():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    from geode_b200 import cuda_lib
    L = cuda_lib()
    L.gcuda_debug_expf_table.restype = C.c_int
    L.gcuda_debug_expf_table.argtypes = [C.c_uint32, C.c_int64, C.c_void_p, C.c_void_p]
    O = op.oracle_lib()
    chunk = 1 << 28
    dev = torch.empty(chunk, dtype=torch.float32, device="cuda")
    host = torch.empty(chunk, dtype=torch.float32, pin_memory=True)
    threads = max(1, min(32, os.cpu_count() or 1))
    first = np.zeros(16, np.uint32)
    bad = 0
    for lo in range(0, 1 << 32, chunk):
        assert L.gcuda_debug_expf_table(lo, chunk, dev.data_ptr(), None) == 0
        host.copy_(dev)
        bad += O.go_expf_check_table(lo, chunk, host.data_ptr(), threads, first.ctypes.data, 16)
    assert bad == 0, (bad, [hex(int(b)) for b in first[: min(bad, 16)]])
