"""The C ABI's edge cases on the GPU: every bad call returns its error and leaves the handle usable and the
conversation as it was - a verified batch of 0 or more than max_tokens tokens, a token id out of range (checked
before anything runs, as the engine checks its embedding rows, engine/src/model.cpp:1551-1555), keeping 0 or all
rows, accepting before any batch, a batch past the end of the context, the operators' sizes out of range. After the
refusals the handle's next batch equals, bit for bit, that of a second handle that saw only the good calls."""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from geode_b200 import cuda_lib, synth  # noqa: E402

pytestmark = pytest.mark.gpu

E_ARG, E_STATE = -1, -5


def test_bad_calls_leave_the_conversation(tmp_path):
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    from geode_b200.backend import Backend, GSampling
    shape = synth.tiny_shape("qwen35moe", n_layers=4, ctx=640)
    d = str(tmp_path / "pack")
    synth.write_pack(d, shape, seed=12)
    a = Backend(d, context=40, max_tokens=5)
    b = Backend(d, context=40, max_tokens=5)
    L = a.L
    V = shape.vocab
    try:
        rng = np.random.default_rng(2)
        toks = rng.integers(0, V, 5).astype(np.int32)
        out = np.zeros((5, V), np.float32)
        sp = GSampling(0.0, 1.0, 0)
        kept, nxt = C.c_int(0), C.c_int(0)
        assert L.gcuda_accept(a.g, C.byref(sp), None, None, 0, None, 0, C.byref(kept), C.byref(nxt), None) == E_STATE
        assert L.gcuda_verify(a.g, toks.ctypes.data, 0, out.ctypes.data, None) == E_ARG
        assert L.gcuda_verify(a.g, toks.ctypes.data, 6, out.ctypes.data, None) == E_ARG
        for bad in (V, -1):
            t2 = toks.copy()
            t2[3] = bad
            assert L.gcuda_verify(a.g, t2.ctypes.data, 5, out.ctypes.data, None) == E_ARG
            assert "embedding of token" in a.error()
        assert a.pos == 0
        got_a, _ = a.verify(toks)
        got_b, _ = b.verify(toks)
        assert np.array_equal(got_a, got_b)
        for k in (0, 5):
            assert L.gcuda_keep(a.g, k) == E_ARG
        a.keep(2)
        b.keep(2)
        # past the end of the context (40 positions): refused, nothing moved
        for _ in range(7):
            t = rng.integers(0, V, 5).astype(np.int32)
            ga, _ = a.verify(t)
            gb, _ = b.verify(t)
            assert np.array_equal(ga, gb)
        assert a.pos == 37
        assert L.gcuda_verify(a.g, toks.ctypes.data, 5, out.ctypes.data, None) == E_ARG
        assert a.pos == 37
        t = rng.integers(0, V, 3).astype(np.int32)
        ga, _ = a.verify(t)
        gb, _ = b.verify(t)
        assert np.array_equal(ga, gb) and a.pos == b.pos == 40
    finally:
        a.close()
        b.close()
    # the operators' refusals (nothing launched)
    Lc = cuda_lib()
    x = torch.zeros(16, device="cuda")
    assert Lc.gcuda_op_greedy_verify(x.data_ptr(), x.data_ptr(), 0, 4, 8, x.data_ptr(), x.data_ptr(), x.data_ptr(),
                                     None) != 0
    assert Lc.gcuda_op_greedy_verify(x.data_ptr(), x.data_ptr(), 20000, 4, 8, x.data_ptr(), x.data_ptr(), x.data_ptr(),
                                     None) != 0   # (more rows than the grid's y dimension)
