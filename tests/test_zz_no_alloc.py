"""gcuda_op_spec_reject_static (the rejection-sampling operator whose scratch is a fixed device array of the library,
for callers that must not allocate device memory at call time) against gcuda_spec_reject (the handle's entry point,
which allocates its scratch) on the same inputs: the same accepted lengths and next tokens, on two calls in a row.
Collected last (file name), so it runs both alone and after the other tests in one process."""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from geode_b200 import cuda_lib  # noqa: E402
from geode_b200.backend import GSampling, _sig  # noqa: E402

pytestmark = pytest.mark.gpu


def _inputs(seed, S, k, V):
    rng = np.random.default_rng(seed)
    target = (rng.standard_normal((S, k + 1, V)) * 3).astype(np.float32)
    draft = target[:, :k, :] + (rng.standard_normal((S, k, V)) * 0.3).astype(np.float32)
    drafts = np.argmax(draft, axis=2).astype(np.int32)
    drafts[::3, 1] = rng.integers(0, V, len(drafts[::3]))
    return target, np.ascontiguousarray(draft), np.ascontiguousarray(drafts)


def test_static_scratch_matches_allocating_entry():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    L = cuda_lib()
    _sig(L)
    L.gcuda_op_spec_reject_static.restype = C.c_int
    L.gcuda_op_spec_reject_static.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p,
                                              C.c_uint64, C.c_void_p, C.c_void_p, C.c_void_p]
    err = C.create_string_buffer(256)
    g = L.gcuda_open(0, err, 256)
    assert g, err.value
    try:
        sp = GSampling(0.7, 0.95, 20)
        for call, (S, k, V) in enumerate([(40, 4, 8192), (7, 8, 3000)]):   # two calls in a row, different sizes
            target, draft, drafts = _inputs(100 + call, S, k, V)
            d_t = torch.from_numpy(target).cuda()
            d_d = torch.from_numpy(draft).cuda()
            acc_a, nxt_a = np.zeros(S, np.int32), np.zeros(S, np.int32)
            acc_b, nxt_b = np.full(S, -7, np.int32), np.full(S, -7, np.int32)
            assert L.gcuda_spec_reject(g, d_t.data_ptr(), d_d.data_ptr(), drafts.ctypes.data, S, k, V, C.byref(sp), 99,
                                       acc_a.ctypes.data, nxt_a.ctypes.data) == 0
            stream = torch.cuda.current_stream().cuda_stream
            assert L.gcuda_op_spec_reject_static(d_t.data_ptr(), d_d.data_ptr(), drafts.ctypes.data, S, k, V, C.byref(sp),
                                                 99, acc_b.ctypes.data, nxt_b.ctypes.data, stream) == 0
            assert np.array_equal(acc_a, acc_b) and np.array_equal(nxt_a, nxt_b), call
            assert (nxt_b >= 0).all()
        # beyond the fixed scratch: refused, nothing launched
        target, draft, drafts = _inputs(7, 2, 17, 64)
        d_t, d_d = torch.from_numpy(target).cuda(), torch.from_numpy(draft).cuda()
        a, n = np.zeros(2, np.int32), np.zeros(2, np.int32)
        assert L.gcuda_op_spec_reject_static(d_t.data_ptr(), d_d.data_ptr(), drafts.ctypes.data, 2, 17, 64, C.byref(sp), 1,
                                             a.ctypes.data, n.ctypes.data, None) != 0
    finally:
        L.gcuda_close(g)
