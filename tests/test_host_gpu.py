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
    _fields_ = [("temperature", C.c_float), ("top_p", C.c_float), ("top_k", C.c_int32), ("seed", C.c_uint64),
                ("presence_penalty", C.c_float)]


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


def test_host_presence_steps(env):
    """ghost_step with geode_generate's presence penalty over consecutive steps of one answer: the host keeps the
    answer's tokens (batch[0], then every row it samples) from ghost_set_sampling on; each step's kept and next equal
    the oracle's rule (go_accept_seen) on the same logits with the oracle's own list carried along, greedy and
    sampled."""
    H, m, d, shape = env
    from geode_b200.backend import Backend
    be = Backend(d, context=shape.ctx, max_tokens=5)
    O = op.oracle_lib()
    rng = np.random.default_rng(12)
    err = C.create_string_buffer(512)
    H.ghost_reset.argtypes = [C.c_void_p, C.c_char_p, C.c_size_t]
    H.ghost_prefill.argtypes = [C.c_void_p, C.c_void_p, C.c_int32, C.c_char_p, C.c_size_t]
    try:
        # both handles at the same conversation: the host's position, reached by a prefill on the Python handle
        assert H.ghost_reset(m, err, 512) == 0, err.value
        prompt = rng.integers(0, shape.vocab, 7).astype(np.int32)
        assert H.ghost_prefill(m, prompt.ctypes.data_as(C.c_void_p), 7, err, 512) == 0, err.value
        be.reset()
        be.verify(prompt[:5])
        be.verify(prompt[5:])
        for temp, seed, pen in [(0.0, 0, 2.0), (0.8, 91, 1.25)]:
            sp = GSamp(temp, 0.95 if temp else 1.0, 40 if temp else 0, seed, pen)
            assert H.ghost_set_sampling(m, C.byref(sp)) == 0
            seen = []
            mt_seed = seed   # the host's sampler stream: one draw per sampled row, from the seed on
            draws = 0
            tok = int(rng.integers(0, shape.vocab))
            for step in range(4):
                batch = np.array([tok] + [int(t) for t in rng.integers(0, shape.vocab, 4)], np.int32)
                rows, _ = be.verify(batch)
                if tok not in seen:
                    seen.append(tok)
                u_all = op.oracle_uniforms(O, mt_seed, draws + 5)
                kept_r, next_r, samples_r, seen_after = _accept_with_stream(O, rows, batch, temp, sp, u_all[draws:],
                                                                            pen, seen)
                kept, nxt = C.c_int32(0), C.c_int32(0)
                assert H.ghost_step(m, batch.ctypes.data_as(C.c_void_p), 5, None, 0, C.byref(kept), C.byref(nxt), err,
                                    512) == 0, err.value
                assert (kept.value, nxt.value) == (kept_r, next_r), (temp, step, kept.value, nxt.value, kept_r, next_r)
                seen = seen_after
                draws += kept_r if temp > 0 else 0
                if kept.value < 5:
                    be.keep(kept.value)
                assert H.ghost_position(m) == be.pos
                tok = nxt.value
    finally:
        be.close()
        H.ghost_reset(m, err, 512)   # (the conversation empty again for the tests after this one)


def _accept_with_stream(O, rows, batch, temp, sp, u, pen, seen):
    """go_accept_seen's rule with the given uniforms in place of a seeded stream: row by row, go_sample on the
    penalised row (the oracle's own go_sample, pinned to the reference's Sampler)."""
    rows = np.ascontiguousarray(rows, dtype=np.float32)
    V = rows.shape[1]
    seen = list(seen)
    kept, samples = 1, []
    for i in range(5):
        r = rows[i].copy()
        idx = np.array(seen, np.int64)
        if pen != 0.0 and idx.size:
            r[idx] = r[idx] - np.float32(pen)
        y = O.go_sample(r.ctypes.data, V, sp.temperature, sp.top_p, sp.top_k, float(u[i]) if temp > 0 else 0.0)
        samples.append(y)
        if pen != 0.0 and y not in seen:
            seen.append(y)
        if i + 1 < 5 and y == batch[i + 1]:
            kept += 1
            continue
        return kept, y, samples, seen
    return kept, -1, samples, seen


def test_host_state_file(env, tmp_path):
    """ghost_state_save / ghost_state_load through the device, in the engine's own state file: a state the reference
    engine saved (oracle/_ref, where it is built; else one written from the oracle's state by ghost_state_write) loads
    into the GPU, whose next batch then matches the oracle's continuation within the parity tolerance; the GPU's state
    saved back reads as the same buffers (ghost_state_read) and loads again; a file of another model is refused and
    leaves the conversation empty."""
    H, m, d, shape = env
    from test_state_file import Shapes, _state
    H.ghost_state_save.argtypes = [C.c_void_p, C.c_char_p, C.c_int32, C.POINTER(C.c_int32), C.c_char_p, C.c_size_t]
    H.ghost_state_load.argtypes = [C.c_void_p, C.c_char_p, C.POINTER(C.c_int32), C.c_char_p, C.c_size_t]
    H.ghost_pending.argtypes = [C.c_void_p]
    H.ghost_state_fingerprint.restype = C.c_uint64
    H.ghost_state_fingerprint.argtypes = [C.c_char_p, C.POINTER(Shapes)]
    H.ghost_state_write.argtypes = [C.c_char_p, C.c_uint64, C.POINTER(Shapes), C.c_int32, C.c_int32, C.c_uint64,
                                    C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int32, C.c_char_p,
                                    C.c_size_t]
    H.ghost_state_peek.argtypes = [C.c_char_p, C.c_uint64, C.POINTER(Shapes), C.c_int32, C.POINTER(C.c_int32),
                                   C.POINTER(C.c_int32), C.POINTER(C.c_uint64), C.c_char_p, C.c_size_t]
    H.ghost_state_read.argtypes = [C.c_char_p, C.c_uint64, C.POINTER(Shapes), C.c_int32, C.c_void_p, C.c_void_p,
                                   C.c_void_p, C.c_void_p, C.c_void_p, C.POINTER(C.c_int32), C.c_char_p, C.c_size_t]
    ora = op.Oracle(d)
    c = ora.cfg
    conv_dim = 2 * c.gdn_k_heads * c.gdn_k_dim + c.gdn_v_heads * c.gdn_v_dim
    s = Shapes(ora.n_attn, c.n_kv_heads, c.n_kv_heads * c.head_dim, c.hidden, c.n_layers,
               ora.n_gdn * conv_dim * (c.conv_kernel - 1), ora.n_gdn * c.gdn_v_heads * c.gdn_k_dim * c.gdn_v_dim)
    fp = H.ghost_state_fingerprint(d.encode(), C.byref(s))
    rng = np.random.default_rng(8)
    prompt = rng.integers(0, shape.vocab, 260).astype(np.int32)
    err = C.create_string_buffer(512)
    a = str(tmp_path / "a.state")
    if op.have_reference():
        ref = op.Reference(d, ctx=shape.ctx)
        ref.forward(prompt, all_logits=False)
        ref.save_state(a)
        ref.close()
    else:
        st0, kv0, kvs0 = _state(ora, prompt, shape.ctx)
        assert H.ghost_state_write(a.encode(), fp, C.byref(s), st0.pos, 0, 9, st0.conv.ctypes.data, st0.gdn.ctypes.data,
                                   kv0.ctypes.data, kvs0.ctypes.data, None, 0, err, 512) == 0, err.value
    pos = C.c_int32(0)
    assert H.ghost_state_load(m, a.encode(), C.byref(pos), err, 512) == 0, err.value
    assert pos.value == 260 and H.ghost_position(m) == 260 and H.ghost_pending(m) == 0
    st, _, _ = _state(ora, prompt, shape.ctx)
    toks = rng.integers(0, shape.vocab, 5).astype(np.int32)
    lg = np.zeros((5, shape.vocab), np.float32)
    assert H.ghost_verify(m, toks.ctypes.data_as(C.c_void_p), 5, lg.ctypes.data_as(C.c_void_p), err, 512) == 0, err.value
    want = ora.forward(st, toks)["logits"]
    span = want.max(1) - want.min(1)
    assert np.all(np.abs(lg - want).max(1) <= 1e-2 * span)
    # the GPU's state (265 positions) saved, read back on the host, loaded again
    b = str(tmp_path / "b.state")
    assert H.ghost_state_save(m, b.encode(), 0, C.byref(pos), err, 512) == 0, err.value
    assert pos.value == 265
    from test_state_file import _read
    rc, e, got = _read(H, b, fp, s, shape.ctx)
    assert rc == 0, e
    P, extra, cid, conv, gdn, kv, kvs = got
    assert P == 265
    assert np.allclose(gdn[:st.gdn.size], st.gdn, rtol=5e-2, atol=5e-3)
    assert np.abs(kv.astype(np.int32) - _state(ora, np.concatenate([prompt, toks]), shape.ctx)[1].astype(np.int32)).max() <= 2
    assert H.ghost_state_load(m, b.encode(), C.byref(pos), err, 512) == 0, err.value
    assert H.ghost_position(m) == 265
    lg2 = np.zeros((5, shape.vocab), np.float32)
    toks2 = rng.integers(0, shape.vocab, 5).astype(np.int32)
    assert H.ghost_verify(m, toks2.ctypes.data_as(C.c_void_p), 5, lg2.ctypes.data_as(C.c_void_p), err, 512) == 0
    want2 = ora.forward(st, toks2)["logits"]
    span2 = want2.max(1) - want2.min(1)
    assert np.all(np.abs(lg2 - want2).max(1) <= 1e-2 * span2)
    # another model's file: refused, the conversation empty
    bad = bytearray(open(b, "rb").read())
    bad[16] ^= 1   # (the fingerprint; the checksum no longer matches either)
    open(str(tmp_path / "bad.state"), "wb").write(bad)
    assert H.ghost_state_load(m, str(tmp_path / "bad.state").encode(), C.byref(pos), err, 512) == 3
    assert H.ghost_position(m) == 0 and H.ghost_pending(m) == -1


def test_host_state_file_mtp(tmp_path):
    """A pack with the MTP layer through ghost_state_save / ghost_state_load: after five verified batches, each with
    the MTP pass over its rows drafted from the device (hidden NULL), the saved file holds the model's and the MTP layer's KV and the last hidden row, which are the oracle's after the
    same tokens within the parity tolerance; loaded back, a draft with hidden NULL takes the loaded row and equals
    the draft made before the save from the file's row, bit for bit (the same kernels on the same state)."""
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    from test_state_file import Shapes, _read
    H = C.CDLL(HOST_SO)
    vp, i32 = C.c_void_p, C.c_int32
    H.ghost_open.argtypes = [C.c_char_p, i32, i32, i32, C.POINTER(vp), C.c_char_p, C.c_size_t]
    H.ghost_close.argtypes = [vp]
    H.ghost_position.argtypes = [vp]
    H.ghost_verify.argtypes = [vp, vp, i32, vp, C.c_char_p, C.c_size_t]
    H.ghost_draft.argtypes = [vp, vp, i32, i32, vp, C.POINTER(i32), C.POINTER(C.c_float), C.c_char_p, C.c_size_t]
    H.ghost_state_save.argtypes = [vp, C.c_char_p, i32, C.POINTER(i32), C.c_char_p, C.c_size_t]
    H.ghost_state_load.argtypes = [vp, C.c_char_p, C.POINTER(i32), C.c_char_p, C.c_size_t]
    H.ghost_state_fingerprint.restype = C.c_uint64
    H.ghost_state_fingerprint.argtypes = [C.c_char_p, C.POINTER(Shapes)]
    H.ghost_state_peek.argtypes = [C.c_char_p, C.c_uint64, C.POINTER(Shapes), i32, C.POINTER(i32), C.POINTER(i32),
                                   C.POINTER(C.c_uint64), C.c_char_p, C.c_size_t]
    H.ghost_state_read.argtypes = [C.c_char_p, C.c_uint64, C.POINTER(Shapes), i32, vp, vp, vp, vp, vp, C.POINTER(i32),
                                   C.c_char_p, C.c_size_t]
    shape = synth.tiny_shape("qwen35moe", n_layers=4, ctx=640)
    d = str(tmp_path / "mtp")
    synth.write_pack(d, shape, seed=81, mtp=True)
    ora = op.Oracle(d)
    c = ora.cfg
    conv_dim = 2 * c.gdn_k_heads * c.gdn_k_dim + c.gdn_v_heads * c.gdn_v_dim
    A, row = ora.n_attn + 1, c.n_kv_heads * c.head_dim
    s = Shapes(A, c.n_kv_heads, row, c.hidden, c.n_layers, ora.n_gdn * conv_dim * (c.conv_kernel - 1),
               ora.n_gdn * c.gdn_v_heads * c.gdn_k_dim * c.gdn_v_dim, 1)
    fp = H.ghost_state_fingerprint(d.encode(), C.byref(s))
    toks = np.random.default_rng(82).integers(0, shape.vocab, 26).astype(np.int32)
    err = C.create_string_buffer(512)
    m = C.c_void_p()
    assert H.ghost_open(d.encode(), 0, shape.ctx, 5, C.byref(m), err, 512) == 0, err.value
    try:
        dh, ph = i32(0), C.c_float(0.0)
        for p0 in range(0, 25, 5):
            assert H.ghost_verify(m, toks[p0:].ctypes.data_as(vp), 5, None, err, 512) == 0, err.value
            nxt = np.ascontiguousarray(toks[p0 + 1:p0 + 6])
            assert H.ghost_draft(m, nxt.ctypes.data_as(vp), 5, p0, None, C.byref(dh), C.byref(ph), err, 512) == 0, \
                err.value
        a = str(tmp_path / "a.state")
        pos = i32(0)
        assert H.ghost_state_save(m, a.encode(), 0, C.byref(pos), err, 512) == 0, err.value
        assert pos.value == 25
        rc, e, got = _read(H, a, fp, s, shape.ctx, with_hidden=True)
        assert rc == 0, e
        P, extra, cid, conv, gdn, kv, kvs, hrow = got
        assert P == 25 and hrow is not None
        # the oracle after the same tokens (its hidden rows feed its MTP passes)
        st = ora.new_state(shape.ctx)
        hid = ora.forward(st, toks[:25], logits=False, hidden=True)["hidden"]
        span = hid[24].max() - hid[24].min()
        assert np.abs(hrow - hid[24]).max() <= 1e-2 * span
        for p0 in range(0, 25, 5):
            ora.forward_mtp(st, toks[p0 + 1:p0 + 6], hid[p0:p0 + 5], p0, logits=False)
        kv_o = st.kv.reshape(A - 1, 2, shape.ctx, row)[:, :, :25]
        assert np.abs(kv[:A - 1].astype(np.int32) - kv_o.astype(np.int32)).max() <= 2
        mkv_o = st.mtp_kv.reshape(2, shape.ctx, row)[:, :25]
        assert np.abs(kv[A - 1].astype(np.int32) - mkv_o.astype(np.int32)).max() <= 2
        # the draft from the file's row, then loaded: the draft from the loaded row (hidden NULL) is the same
        t25 = np.ascontiguousarray(toks[25:26])
        d1, p1 = i32(0), C.c_float(0.0)
        assert H.ghost_draft(m, t25.ctypes.data_as(vp), 1, 24, hrow.ctypes.data_as(vp), C.byref(d1), C.byref(p1), err,
                             512) == 0, err.value
        assert H.ghost_state_load(m, a.encode(), C.byref(pos), err, 512) == 0, err.value
        assert pos.value == 25 and H.ghost_position(m) == 25
        d2, p2 = i32(0), C.c_float(0.0)
        assert H.ghost_draft(m, t25.ctypes.data_as(vp), 1, 24, None, C.byref(d2), C.byref(p2), err, 512) == 0, err.value
        assert (d1.value, np.float32(p1.value)) == (d2.value, np.float32(p2.value))
    finally:
        H.ghost_close(m)


def test_host_prefill_mtp(tmp_path):
    """ghost_prefill on a pack with the MTP layer runs the layer over the prompt as the engine's prompt does
    (engine/src/geode.cpp:132-150): the first draft afterwards - the pending token at the last position, hidden NULL -
    equals the Python binding's replay of the same calls bit for bit, and its logits are the oracle's (its MTP passes
    over every prompt position fed the GPU's hidden rows) within the parity tolerance."""
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    from geode_b200.backend import Backend
    H = C.CDLL(HOST_SO)
    vp, i32 = C.c_void_p, C.c_int32
    H.ghost_open.argtypes = [C.c_char_p, i32, i32, i32, C.POINTER(vp), C.c_char_p, C.c_size_t]
    H.ghost_close.argtypes = [vp]
    H.ghost_prefill.argtypes = [vp, vp, i32, C.c_char_p, C.c_size_t]
    H.ghost_draft.argtypes = [vp, vp, i32, i32, vp, C.POINTER(i32), C.POINTER(C.c_float), C.c_char_p, C.c_size_t]
    shape = synth.tiny_shape("qwen35moe", n_layers=4, ctx=640)
    d = str(tmp_path / "mtp")
    synth.write_pack(d, shape, seed=83, mtp=True)
    toks = np.random.default_rng(84).integers(0, shape.vocab, 24).astype(np.int32)
    P = 23
    err = C.create_string_buffer(512)
    m = C.c_void_p()
    assert H.ghost_open(d.encode(), 0, shape.ctx, 5, C.byref(m), err, 512) == 0, err.value
    try:
        assert H.ghost_prefill(m, toks.ctypes.data_as(vp), P, err, 512) == 0, err.value
        dh, ph = i32(0), C.c_float(0.0)
        nxt = np.ascontiguousarray(toks[P:P + 1])
        assert H.ghost_draft(m, nxt.ctypes.data_as(vp), 1, P - 1, None, C.byref(dh), C.byref(ph), err, 512) == 0, \
            err.value
    finally:
        H.ghost_close(m)
    # the same calls through the Python binding
    be = Backend(d, context=shape.ctx, max_tokens=5)
    hid = np.zeros((P, shape.hidden), np.float32)
    for i in range(0, P, 5):
        k = min(5, P - i)
        _, hid[i:i + k] = be.verify(toks[i:i + k], logits=False, hidden=True)
        if i:
            be.draft(toks[i:i + 1], i - 1, hidden=hid[i - 1:i])
        if k > 1:
            be.draft(toks[i + 1:i + k], i)
    dp, pp, lg = be.draft(nxt, P - 1, hidden=hid[P - 1:P], logits=True)
    be.close()
    assert (dh.value, np.float32(ph.value)) == (dp, np.float32(pp)), (dh.value, dp, ph.value, pp)
    # the oracle: its MTP passes over the prompt's positions with the GPU's rows, then the draft position
    ora = op.Oracle(d)
    st = ora.new_state(shape.ctx)
    ora.forward(st, toks[:P], logits=False)
    for p0 in range(0, P - 1, 5):
        p1 = min(p0 + 5, P - 1)
        ora.forward_mtp(st, toks[p0 + 1:p1 + 1], hid[p0:p1], p0, logits=False)
    want, _ = ora.forward_mtp(st, nxt, hid[P - 1:P], P - 1)
    assert np.abs(lg - want).max() <= 1e-2 * (want.max() - want.min())


def test_host_prefill(env):
    """ghost_prefill (geode_prefill's counterpart): a 23-token prompt in through the verify step, then a batch whose
    logits match the oracle's after the same prompt within the parity tolerance; a token out of range is refused."""
    H, m, d, shape = env
    H.ghost_prefill.argtypes = [C.c_void_p, C.c_void_p, C.c_int32, C.c_char_p, C.c_size_t]
    H.ghost_pending.argtypes = [C.c_void_p]
    err = C.create_string_buffer(512)
    ora = op.Oracle(d)
    st = ora.new_state(shape.ctx)
    rng = np.random.default_rng(21)
    p0 = H.ghost_position(m)
    if p0:   # (the conversation the earlier tests left: the oracle replays from empty, so start from empty too)
        pytest.skip("the shared handle holds a conversation")
    prompt = rng.integers(0, shape.vocab, 23).astype(np.int32)
    assert H.ghost_prefill(m, prompt.ctypes.data_as(C.c_void_p), 23, err, 512) == 0, err.value
    assert H.ghost_position(m) == 23 and H.ghost_pending(m) == -1
    ora.forward(st, prompt, logits=False)
    toks = rng.integers(0, shape.vocab, 5).astype(np.int32)
    lg = np.zeros((5, shape.vocab), np.float32)
    assert H.ghost_verify(m, toks.ctypes.data_as(C.c_void_p), 5, lg.ctypes.data_as(C.c_void_p), err, 512) == 0, err.value
    want = ora.forward(st, toks)["logits"]
    span = want.max(1) - want.min(1)
    assert np.all(np.abs(lg - want).max(1) <= 1e-2 * span)
    bad = prompt[:3].copy()
    bad[1] = shape.vocab
    assert H.ghost_prefill(m, bad.ctypes.data_as(C.c_void_p), 3, err, 512) == 1
    assert H.ghost_position(m) == 28
    # ghost_reset: the conversation empty; the same prompt again gives the same next batch
    H.ghost_reset.argtypes = [C.c_void_p, C.c_char_p, C.c_size_t]
    assert H.ghost_reset(m, err, 512) == 0 and H.ghost_position(m) == 0 and H.ghost_pending(m) == -1
    assert H.ghost_prefill(m, prompt.ctypes.data_as(C.c_void_p), 23, err, 512) == 0, err.value
    lg2 = np.zeros_like(lg)
    assert H.ghost_verify(m, toks.ctypes.data_as(C.c_void_p), 5, lg2.ctypes.data_as(C.c_void_p), err, 512) == 0
    assert np.array_equal(lg2, lg)


@pytest.mark.parametrize("vocab_file", [False, True])
def test_host_drafts(tmp_path, vocab_file):
    """ghost_draft / ghost_draft_next through the host (a pack with the MTP layer: CudaModel adopts mtp.* and the
    MTP layer's experts, gcuda_set_mtp) equal the Python binding's gcuda_draft / gcuda_draft_next after the same
    batches - the same kernels on the same bytes, so the same drafts and probabilities bit for bit; the pass's
    numerics against the oracle are tests/test_mtp_gpu.py's. With a draft vocabulary (draft_vocab.bin) both sides
    build the same draft head and every draft is one of its ids. A pack without the layer refuses to draft."""
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    from geode_b200.backend import Backend
    H = C.CDLL(HOST_SO)
    vp, i32 = C.c_void_p, C.c_int32
    H.ghost_open.argtypes = [C.c_char_p, i32, i32, i32, C.POINTER(vp), C.c_char_p, C.c_size_t]
    H.ghost_close.argtypes = [vp]
    H.ghost_verify.argtypes = [vp, vp, i32, vp, C.c_char_p, C.c_size_t]
    H.ghost_draft.argtypes = [vp, vp, i32, i32, vp, C.POINTER(i32), C.POINTER(C.c_float), C.c_char_p, C.c_size_t]
    H.ghost_draft_next.argtypes = [vp, i32, i32, C.POINTER(i32), C.POINTER(C.c_float), C.c_char_p, C.c_size_t]
    shape = synth.tiny_shape("qwen35moe", n_layers=4, ctx=640)
    d = str(tmp_path / "mtp")
    synth.write_pack(d, shape, seed=71, mtp=True)
    rng = np.random.default_rng(72)
    ids = None
    if vocab_file:
        ids = set(int(i) for i in rng.choice(shape.vocab, 70, replace=False))
        synth.write_draft_vocab(d, sorted(ids))
    err = C.create_string_buffer(512)
    m = C.c_void_p()
    assert H.ghost_open(d.encode(), 0, shape.ctx, 5, C.byref(m), err, 512) == 0, err.value
    be = Backend(d, context=shape.ctx, max_tokens=5)
    assert be.L.gcuda_draft_rows(be.g) == (96 if vocab_file else shape.vocab)
    try:
        pos = 0
        tok = int(rng.integers(0, shape.vocab))
        for rep in range(3):
            batch = np.array([tok] + [int(t) for t in rng.integers(0, shape.vocab, 4)], np.int32)
            assert H.ghost_verify(m, batch.ctypes.data_as(vp), 5, None, err, 512) == 0, err.value
            be.verify(batch, logits=False)
            nxt = np.array(list(batch[1:]) + [int(rng.integers(0, shape.vocab))], np.int32)
            dh, ph = i32(0), C.c_float(0.0)
            assert H.ghost_draft(m, nxt.ctypes.data_as(vp), 5, pos, None, C.byref(dh), C.byref(ph), err, 512) == 0, \
                err.value
            dp, pp, _ = be.draft(nxt, pos)
            assert (dh.value, np.float32(ph.value)) == (dp, np.float32(pp)), (rep, dh.value, dp, ph.value, pp)
            assert ids is None or dp in ids
            q = pos + 5
            assert H.ghost_draft_next(m, dh.value, q, C.byref(dh), C.byref(ph), err, 512) == 0, err.value
            dp, pp, _ = be.draft_next(dp, q)
            assert (dh.value, np.float32(ph.value)) == (dp, np.float32(pp))
            pos += 5
            tok = dh.value
    finally:
        H.ghost_close(m)
        be.close()
    plain = str(tmp_path / "plain")
    synth.write_pack(plain, shape, seed=71)
    assert H.ghost_open(plain.encode(), 0, shape.ctx, 5, C.byref(m), err, 512) == 0, err.value
    try:
        toks = np.array([1, 2], np.int32)
        dh, ph = i32(0), C.c_float(0.0)
        hid = np.zeros((2, shape.hidden), np.float32)
        assert H.ghost_draft(m, toks.ctypes.data_as(vp), 2, 0, hid.ctypes.data_as(vp), C.byref(dh), C.byref(ph), err,
                             512) != 0
        assert b"MTP" in err.value
    finally:
        H.ghost_close(m)
