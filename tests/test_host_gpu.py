"""The C++ host side on the GPU (libgeode_host.so over libgeode_cuda.so): a pack opened by the host gives the same
logits as the Python binding of the backend (the same kernels on the same bytes), within the parity tolerance of the
oracle, and its speculation step (verify, the engine's acceptance rule with the sampler's mt19937_64 stream, rollback)
equals the oracle's rule on those logits, greedy and sampled."""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from geode_b200 import synth  # noqa: E402
import oracle_py as op  # noqa: E402
from test_host import HOST_SO  # noqa: E402

pytestmark = pytest.mark.gpu


class GSamp(C.Structure):
    _fields_ = [("temperature", C.c_float), ("top_p", C.c_float), ("top_k", C.c_int32), ("seed", C.c_uint64)]


@pytest.fixture(scope="module")
def env(tmp_path_factory):
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    H = C.CDLL(HOST_SO)
    H.ghost_open.argtypes = [C.c_char_p, C.c_int32, C.c_int32, C.c_int32, C.POINTER(C.c_void_p), C.c_char_p, C.c_size_t]
    H.ghost_close.argtypes = [C.c_void_p]
    H.ghost_position.argtypes = [C.c_void_p]
    d = str(tmp_path_factory.mktemp("hostpack"))
    shape = synth.tiny_shape("qwen35moe", n_layers=4, ctx=640)
    synth.write_pack(d, shape, seed=4)
    m = C.c_void_p()
    err = C.create_string_buffer(512)
    assert H.ghost_open(d.encode(), 0, shape.ctx, 5, C.byref(m), err, 512) == 0, err.value
    yield H, m, d, shape
    H.ghost_close(m)


def test_host_verify_and_steps(env):
    H, m, d, shape = env
    from geode_b200.backend import Backend
    be = Backend(d, context=shape.ctx, max_tokens=5)
    ora = op.Oracle(d)
    st = ora.new_state(shape.ctx)
    lib = op.oracle_lib()
    rng = np.random.default_rng(3)
    err = C.create_string_buffer(512)
    try:
        toks = rng.integers(0, shape.vocab, 5).astype(np.int32)
        lg = np.zeros((5, shape.vocab), np.float32)
        assert H.ghost_verify(m, toks.ctypes.data_as(C.c_void_p), 5, lg.ctypes.data_as(C.c_void_p), err, 512) == 0, err.value
        ref_py, _ = be.verify(toks)
        assert np.array_equal(lg, ref_py)   # the same kernels, the same bytes
        ref = ora.forward(st, toks)["logits"]
        span = ref.max(1) - ref.min(1)
        assert np.all(np.abs(lg - ref).max(1) <= 1e-2 * span)
        assert H.ghost_keep(m, 2, err, 512) == 0   # a rollback to two rows on both handles
        be.keep(2)
        assert H.ghost_position(m) == be.pos == 2
        # speculation steps, greedy then sampled: kept / next equal the oracle's rule on the same logits
        for temp, seed in [(0.0, 0), (0.8, 77)]:
            sp = GSamp(temp, 0.95 if temp else 1.0, 40 if temp else 0, seed)
            assert H.ghost_set_sampling(m, C.byref(sp)) == 0
            batch = rng.integers(0, shape.vocab, 5).astype(np.int32)
            rows, _ = be.verify(batch)   # (the Python handle mirrors the host's state: its logits for the rule)
            n = C.c_int(0)
            s = np.zeros(5, np.int32)
            k_ref = lib.go_accept(np.ascontiguousarray(rows).ctypes.data, 5, shape.vocab, batch.ctypes.data, temp,
                                  sp.top_p, sp.top_k, seed, None, 0, C.byref(n), s.ctypes.data)
            kept, nxt = C.c_int32(0), C.c_int32(0)
            assert H.ghost_step(m, batch.ctypes.data_as(C.c_void_p), 5, None, 0, C.byref(kept), C.byref(nxt), err, 512) == 0, err.value
            assert (kept.value, nxt.value) == (k_ref, n.value)
            if kept.value < 5:
                be.keep(kept.value)
            assert H.ghost_position(m) == be.pos
    finally:
        be.close()
