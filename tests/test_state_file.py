"""The engine's state file through the host library, without a GPU (libgeode_host.so: ghost_state_write / peek /
read, the format behind ghost_state_save / ghost_state_load).

- pinned to the reference engine (oracle/_ref, its own Model::save_state / load_state): the file the reference saves
  after a prompt reads back as the oracle's state after the same prompt (bit for bit - the oracle is itself pinned to
  the reference), and the file written here from those buffers equals the reference's byte for byte; a file written
  here loads into the reference, which then continues exactly as the oracle from that state;
- the same pin without the reference build, from tests/golden/state_file.npz (a file the reference saved, with its
  pack's manifest; made by tests/golden/make_golden.py);
- round trip, append (in place: the same buffers back, gen 2, the earlier KV blocks kept), and the refusals: a
  damaged header, another model's fingerprint, a file cut short, an interrupted save, a state longer than the
  context;
- a pack with the MTP layer, pinned to the reference the same way: its file counts the layer's KV slot among the
  attention layers (after them) and the MTP flag in the fingerprint, and keeps the last hidden row (has_hidden).
"""
import ctypes as C
import os

import numpy as np
import pytest

from geode_b200 import synth
import oracle_py as op

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HOST_SO = os.path.join(ROOT, "geode_b200", "libgeode_host.so")
ref_only = pytest.mark.skipif(not op.have_reference(), reason="the reference build oracle/_ref is not here")

OK, E_ARG, E_IO, E_FORMAT = 0, 1, 2, 3


class Shapes(C.Structure):
    _fields_ = [("n_attn", C.c_uint32), ("kv_heads", C.c_uint32), ("kv_row", C.c_uint32), ("hidden", C.c_uint32),
                ("n_layers", C.c_uint32), ("conv_n", C.c_uint64), ("gdn_n", C.c_uint64), ("mtp", C.c_uint32)]


@pytest.fixture(scope="module")
def H():
    if not os.path.exists(HOST_SO):
        pytest.fail(f"{HOST_SO} is not built (python -m geode_b200.build)")
    L = C.CDLL(HOST_SO)
    vp, i32, u64, sz = C.c_void_p, C.c_int32, C.c_uint64, C.c_size_t
    L.ghost_state_fingerprint.restype = u64
    L.ghost_state_fingerprint.argtypes = [C.c_char_p, C.POINTER(Shapes)]
    L.ghost_state_write.argtypes = [C.c_char_p, u64, C.POINTER(Shapes), i32, i32, u64, vp, vp, vp, vp, vp, i32,
                                    C.c_char_p, sz]
    L.ghost_state_peek.argtypes = [C.c_char_p, u64, C.POINTER(Shapes), i32, C.POINTER(i32), C.POINTER(i32),
                                   C.POINTER(u64), C.c_char_p, sz]
    L.ghost_state_read.argtypes = [C.c_char_p, u64, C.POINTER(Shapes), i32, vp, vp, vp, vp, vp, C.POINTER(i32),
                                   C.c_char_p, sz]
    return L


@pytest.fixture(scope="module")
def model(tmp_path_factory):
    shape = synth.tiny_shape("qwen35moe", n_layers=4, ctx=640)
    d = str(tmp_path_factory.mktemp("statepack"))
    synth.write_pack(d, shape, seed=3)
    ora = op.Oracle(d)
    c = ora.cfg
    conv_dim = 2 * c.gdn_k_heads * c.gdn_k_dim + c.gdn_v_heads * c.gdn_v_dim
    s = Shapes(ora.n_attn, c.n_kv_heads, c.n_kv_heads * c.head_dim, c.hidden, c.n_layers,
               ora.n_gdn * conv_dim * (c.conv_kernel - 1), ora.n_gdn * c.gdn_v_heads * c.gdn_k_dim * c.gdn_v_dim)
    toks = np.random.default_rng(4).integers(0, shape.vocab, 400).astype(np.int32)
    return d, shape, ora, s, toks


def _state(ora, toks, ctx):
    st = ora.new_state(ctx)
    ora.forward(st, toks, logits=False)
    c = ora.cfg
    A, row = ora.n_attn, c.n_kv_heads * c.head_dim
    kv = np.ascontiguousarray(st.kv.reshape(A, 2, ctx, row)[:, :, :st.pos])
    kvs = np.ascontiguousarray(st.kvs.reshape(A, 2, ctx, c.n_kv_heads)[:, :, :st.pos])
    return st, kv, kvs


def _p(a):
    return a.ctypes.data


def _write(H, path, fp, s, st, kv, kvs, conv_id=77, extra=-1, append=0, hidden=None):
    err = C.create_string_buffer(256)
    rc = H.ghost_state_write(path.encode(), fp, C.byref(s), st.pos, extra, conv_id, _p(st.conv), _p(st.gdn), _p(kv),
                             _p(kvs), None if hidden is None else _p(hidden), append, err, 256)
    assert rc == OK, err.value
    return rc


def _read(H, path, fp, s, context, with_hidden=False):
    """(rc, error, (position, extra, conversation id, conv, gdn, kv, kv scales[, the hidden row or None]))"""
    err = C.create_string_buffer(256)
    pos, extra, cid = C.c_int32(0), C.c_int32(0), C.c_uint64(0)
    rc = H.ghost_state_peek(path.encode(), fp, C.byref(s), context, C.byref(pos), C.byref(extra), C.byref(cid), err, 256)
    if rc != OK:
        return rc, err.value.decode(), None
    P = pos.value
    conv = np.zeros(max(1, s.conv_n), np.float32)
    gdn = np.zeros(max(1, s.gdn_n), np.float32)
    kv = np.zeros((s.n_attn, 2, P, s.kv_row), np.int8)
    kvs = np.zeros((s.n_attn, 2, P, s.kv_heads), np.float32)
    hid, has = np.zeros(s.hidden, np.float32), C.c_int32(-1)
    rc = H.ghost_state_read(path.encode(), fp, C.byref(s), context, _p(conv), _p(gdn), _p(kv), _p(kvs), _p(hid),
                            C.byref(has), err, 256)
    out = (P, extra.value, cid.value, conv, gdn, kv, kvs)
    return rc, err.value.decode(), out + ((hid if has.value == 1 else None),) if with_hidden else out


def test_roundtrip_append_and_refusals(H, model, tmp_path):
    d, shape, ora, s, toks = model
    fp = H.ghost_state_fingerprint(d.encode(), C.byref(s))
    st1, kv1, kvs1 = _state(ora, toks[:100], shape.ctx)
    st2, kv2, kvs2 = _state(ora, toks[:400], shape.ctx)
    path = str(tmp_path / "a.state")
    _write(H, path, fp, s, st1, kv1, kvs1, extra=123)
    rc, e, got = _read(H, path, fp, s, shape.ctx)
    assert rc == OK, e
    P, extra, cid, conv, gdn, kv, kvs = got
    assert (P, extra, cid) == (100, 123, 77)
    assert np.array_equal(conv[:st1.conv.size], st1.conv) and np.array_equal(gdn[:st1.gdn.size], st1.gdn)
    assert np.array_equal(kv, kv1) and np.array_equal(kvs, kvs1)
    # append: the same conversation grown - written in place, gen 2, and it reads back as the later state
    _write(H, path, fp, s, st2, kv2, kvs2, extra=5, append=1)
    assert not os.path.exists(path + ".tmp")
    raw = open(path, "rb").read()
    assert int.from_bytes(raw[32:40], "little") == 2   # (gen)
    rc, e, got = _read(H, path, fp, s, shape.ctx)
    assert rc == OK, e
    P, extra, cid, conv, gdn, kv, kvs = got
    assert (P, extra, cid) == (400, 5, 77)
    assert np.array_equal(kv, kv2) and np.array_equal(kvs, kvs2) and np.array_equal(gdn[:st2.gdn.size], st2.gdn)
    # the same as a whole write of the later state, but for gen and the header's checksum
    whole = str(tmp_path / "w.state")
    _write(H, whole, fp, s, st2, kv2, kvs2, extra=5)
    raw_w = open(whole, "rb").read()
    assert len(raw) == len(raw_w)
    a, w = np.frombuffer(raw, np.uint8), np.frombuffer(raw_w, np.uint8)
    diff = np.nonzero(a != w)[0]
    assert len(diff) and all(32 <= i < 40 or 136 <= i < 144 or 4096 <= i < 4104 or _in_trail(raw, i) for i in diff)
    # another conversation: not an append (written whole, gen 1)
    _write(H, path, fp, s, st2, kv2, kvs2, conv_id=78, append=1)
    assert int.from_bytes(open(path, "rb").read()[32:40], "little") == 1
    # refusals
    assert _read(H, path, fp + 1, s, shape.ctx)[0] == E_FORMAT            # another model
    assert _read(H, path, fp, s, 400)[0] == E_ARG                          # longer than the context
    bad = bytearray(open(path, "rb").read())
    bad[44] ^= 1                                                           # (extra, under the checksum)
    open(str(tmp_path / "d.state"), "wb").write(bad)
    assert _read(H, str(tmp_path / "d.state"), fp, s, shape.ctx)[0] == E_FORMAT
    good = open(path, "rb").read()
    open(str(tmp_path / "t.state"), "wb").write(good[:len(good) - 1000])
    assert _read(H, str(tmp_path / "t.state"), fp, s, shape.ctx)[0] == E_IO   # cut short
    torn = bytearray(good)
    torn[4096] ^= 1                                                        # (the fixed part's leading gen)
    open(str(tmp_path / "g.state"), "wb").write(torn)
    assert _read(H, str(tmp_path / "g.state"), fp, s, shape.ctx)[0] == E_IO   # an interrupted save
    assert _read(H, str(tmp_path / "missing.state"), fp, s, shape.ctx)[0] == E_IO


def _in_trail(raw, i):
    """i lies in the fixed part's trailing gen (its offset from the header's layout)."""
    fixed_offset = int.from_bytes(raw[104:112], "little")
    fixed_bytes = int.from_bytes(raw[112:120], "little")
    trail = fixed_offset + fixed_bytes - 8
    return trail <= i < trail + 8


@ref_only
def test_pinned_to_the_reference(H, model, tmp_path):
    d, shape, ora, s, toks = model
    fp = H.ghost_state_fingerprint(d.encode(), C.byref(s))
    ref = op.Reference(d, ctx=shape.ctx)
    try:
        ref.forward(toks[:300], all_logits=False)
        a = str(tmp_path / "ref.state")
        ref.save_state(a)
        # the reference's file reads here as the oracle's state after the same prompt
        rc, e, got = _read(H, a, fp, s, shape.ctx)
        assert rc == OK, e
        P, extra, cid, conv, gdn, kv, kvs = got
        st, kv_o, kvs_o = _state(ora, toks[:300], shape.ctx)
        assert P == 300 and extra == 0
        assert np.array_equal(conv[:st.conv.size], st.conv) and np.array_equal(gdn[:st.gdn.size], st.gdn)
        assert np.array_equal(kv, kv_o) and np.array_equal(kvs, kvs_o)
        # written here from those buffers (the reference's conversation id and extra): the same bytes
        b = str(tmp_path / "ours.state")
        _write(H, b, fp, s, st, kv_o, kvs_o, conv_id=cid, extra=0)
        assert open(a, "rb").read() == open(b, "rb").read()
        # a state written here (another length) loads into the reference, which continues as the oracle does
        st2, kv2, kvs2 = _state(ora, toks[:137], shape.ctx)
        c = str(tmp_path / "ours2.state")
        _write(H, c, fp, s, st2, kv2, kvs2, conv_id=5, extra=0)
        ref.load_state(c)
        assert ref.pos == 137
        nxt = toks[137:142]
        got_l = ref.forward(nxt, all_logits=True)["logits"]
        want = ora.forward(st2, nxt, logits=True)["logits"]
        assert np.array_equal(got_l, want)
    finally:
        ref.close()


def test_golden_state_file(H, tmp_path):
    """Without the reference build: tests/golden/state_file.npz holds the file the reference engine's save_state wrote
    after a 20-token prompt on a tiny pack, and that pack's geode.json. The fingerprint computed here from the manifest
    equals the file's; the file reads here as the oracle's state after the same prompt (the pack written again from
    its seed gives the same manifest); written again here from what was read, it is the same bytes."""
    g = np.load(os.path.join(ROOT, "tests", "golden", "state_file.npz"))
    state = g["state"].tobytes()
    d = tmp_path / "pack"
    d.mkdir()
    (d / "geode.json").write_bytes(g["manifest"].tobytes())
    sh = [int(x) for x in g["shapes"]]
    s = Shapes(*sh)
    fp = H.ghost_state_fingerprint(str(d).encode(), C.byref(s))
    assert fp == int.from_bytes(state[16:24], "little")
    path = str(tmp_path / "golden.state")
    open(path, "wb").write(state)
    rc, e, got = _read(H, path, fp, s, 640)
    assert rc == OK, e
    P, extra, cid, conv, gdn, kv, kvs = got
    assert (P, extra) == (20, 0)
    # the oracle's state after the same prompt on the same pack
    shape = synth.tiny_shape("qwen35moe", n_layers=4, ctx=640)
    d2 = str(tmp_path / "again")
    synth.write_pack(d2, shape, seed=int(g["seed"]))
    assert open(os.path.join(d2, "geode.json"), "rb").read() == g["manifest"].tobytes()
    st, kv_o, kvs_o = _state(op.Oracle(d2), g["prompt"], shape.ctx)
    assert np.array_equal(conv[:st.conv.size], st.conv) and np.array_equal(gdn[:st.gdn.size], st.gdn)
    assert np.array_equal(kv, kv_o) and np.array_equal(kvs, kvs_o)
    out = str(tmp_path / "again.state")
    err = C.create_string_buffer(256)
    assert H.ghost_state_write(out.encode(), fp, C.byref(s), P, extra, cid, _p(conv), _p(gdn), _p(kv), _p(kvs), None, 0,
                               err, 256) == OK, err.value
    assert open(out, "rb").read() == state


@ref_only
def test_mtp_state_pinned_to_the_reference(H, tmp_path):
    """A pack with the MTP layer: the reference (drafting on, so its model binds the layer) after a 40-token prompt and
    the MTP layer over the prompt's positions saves a file whose KV holds the main attention layers then the MTP
    layer's slot, and the last position's hidden row; it reads here as the oracle's state after the same prompt and
    passes (the MTP slot's written rows the oracle's MTP KV) with the reference's own hidden row; written again here
    from those buffers it is the same bytes; a file written here loads into the reference, whose next MTP position
    then equals the oracle's bit for bit."""
    shape = synth.tiny_shape("qwen35moe", n_layers=4, ctx=640)
    d = str(tmp_path / "pack")
    synth.write_pack(d, shape, seed=9, mtp=True)
    ora = op.Oracle(d)
    c = ora.cfg
    conv_dim = 2 * c.gdn_k_heads * c.gdn_k_dim + c.gdn_v_heads * c.gdn_v_dim
    A, row, heads = ora.n_attn + 1, c.n_kv_heads * c.head_dim, c.n_kv_heads
    s = Shapes(A, heads, row, c.hidden, c.n_layers, ora.n_gdn * conv_dim * (c.conv_kernel - 1),
               ora.n_gdn * c.gdn_v_heads * c.gdn_k_dim * c.gdn_v_dim, 1)
    s0 = Shapes(A, heads, row, c.hidden, c.n_layers, s.conv_n, s.gdn_n, 0)
    fp = H.ghost_state_fingerprint(d.encode(), C.byref(s))
    assert fp != H.ghost_state_fingerprint(d.encode(), C.byref(s0))   # (the MTP flag is in the fingerprint)
    toks = np.random.default_rng(10).integers(0, shape.vocab, 60).astype(np.int32)
    P = 40
    ref = op.Reference(d, ctx=shape.ctx, draft=True)
    try:
        ref.forward(toks[:P], all_logits=False)
        hid = ref.hidden_rows(P)
        st = ora.new_state(shape.ctx)
        ora.forward(st, toks[:P], logits=False)
        for p0 in range(0, P - 1, 5):
            p1 = min(p0 + 5, P - 1)
            ref.mtp(toks[p0 + 1:p1 + 1], hid[p0:p1], p0, logits=False)
            ora.forward_mtp(st, toks[p0 + 1:p1 + 1], hid[p0:p1], p0, logits=False)
        a = str(tmp_path / "ref.state")
        ref.save_state(a)
        rc, e, got = _read(H, a, fp, s, shape.ctx, with_hidden=True)
        assert rc == OK, e
        pos, extra, cid, conv, gdn, kv, kvs, hrow = got
        assert pos == P and extra == 0
        assert hrow is not None and np.array_equal(hrow, hid[P - 1])
        assert np.array_equal(conv[:st.conv.size], st.conv) and np.array_equal(gdn[:st.gdn.size], st.gdn)
        kv_o = st.kv.reshape(A - 1, 2, shape.ctx, row)[:, :, :P]
        kvs_o = st.kvs.reshape(A - 1, 2, shape.ctx, heads)[:, :, :P]
        assert np.array_equal(kv[:A - 1], kv_o) and np.array_equal(kvs[:A - 1], kvs_o)
        # the MTP slot's rows the passes wrote (positions 0 .. P-2; the engine's forward never writes that slot, so the
        # row at P-1 holds whatever its cache held there - the next MTP pass writes it before anything reads it)
        assert np.array_equal(kv[A - 1][:, :P - 1], st.mtp_kv.reshape(2, shape.ctx, row)[:, :P - 1])
        assert np.array_equal(kvs[A - 1][:, :P - 1], st.mtp_kvs.reshape(2, shape.ctx, heads)[:, :P - 1])
        # written here from those buffers (the reference's conversation id): the same bytes
        b = str(tmp_path / "ours.state")
        _write(H, b, fp, s, st, kv, kvs, conv_id=cid, extra=0, hidden=hrow)
        assert open(a, "rb").read() == open(b, "rb").read()
        # ours loads into the reference, which drafts the next position as the oracle does
        ref.load_state(b)
        assert ref.pos == P
        lg_r, mh_r = ref.mtp(toks[P:P + 1], hrow[None], P - 1)
        lg_o, mh_o = ora.forward_mtp(st, toks[P:P + 1], hrow[None], P - 1)
        assert np.array_equal(lg_r, lg_o) and np.array_equal(mh_r, mh_o)
    finally:
        ref.close()


def test_golden_state_file_mtp(H, tmp_path):
    """Without the reference build, for a pack with the MTP layer: tests/golden/state_file_mtp.npz holds the file the
    reference engine (drafting on) saved after a 20-token prompt and the MTP layer over all its positions, with the
    pack's geode.json and the reference's hidden rows. The fingerprint computed here (the MTP flag in it) equals the
    file's; the file reads here as the oracle's state after the same prompt and passes - the MTP slot after the model's
    attention layers - with the reference's last hidden row; written again here, it is the same bytes."""
    g = np.load(os.path.join(ROOT, "tests", "golden", "state_file_mtp.npz"))
    state = g["state"].tobytes()
    d = tmp_path / "pack"
    d.mkdir()
    (d / "geode.json").write_bytes(g["manifest"].tobytes())
    s = Shapes(*[int(x) for x in g["shapes"]])
    assert s.mtp == 1
    fp = H.ghost_state_fingerprint(str(d).encode(), C.byref(s))
    assert fp == int.from_bytes(state[16:24], "little")
    path = str(tmp_path / "golden.state")
    open(path, "wb").write(state)
    rc, e, got = _read(H, path, fp, s, 640, with_hidden=True)
    assert rc == OK, e
    P, extra, cid, conv, gdn, kv, kvs, hrow = got
    prompt, hid = g["prompt"], g["hidden"]
    assert (P, extra) == (len(prompt), 0)
    assert hrow is not None and np.array_equal(hrow, hid[-1])
    shape = synth.tiny_shape("qwen35moe", n_layers=4, ctx=640)
    d2 = str(tmp_path / "again")
    synth.write_pack(d2, shape, seed=int(g["seed"]), mtp=True)
    assert open(os.path.join(d2, "geode.json"), "rb").read() == g["manifest"].tobytes()
    ora = op.Oracle(d2)
    st = ora.new_state(shape.ctx)
    ora.forward(st, prompt, logits=False)
    ora.forward_mtp(st, np.append(prompt[1:], int(g["next"])), hid, 0, logits=False)
    c = ora.cfg
    A, row, heads = s.n_attn, c.n_kv_heads * c.head_dim, c.n_kv_heads
    assert np.array_equal(conv[:st.conv.size], st.conv) and np.array_equal(gdn[:st.gdn.size], st.gdn)
    assert np.array_equal(kv[:A - 1], st.kv.reshape(A - 1, 2, shape.ctx, row)[:, :, :P])
    assert np.array_equal(kvs[:A - 1], st.kvs.reshape(A - 1, 2, shape.ctx, heads)[:, :, :P])
    assert np.array_equal(kv[A - 1], st.mtp_kv.reshape(2, shape.ctx, row)[:, :P])
    assert np.array_equal(kvs[A - 1], st.mtp_kvs.reshape(2, shape.ctx, heads)[:, :P])
    out = str(tmp_path / "again.state")
    err = C.create_string_buffer(256)
    assert H.ghost_state_write(out.encode(), fp, C.byref(s), P, extra, cid, _p(conv), _p(gdn), _p(kv), _p(kvs),
                                     _p(hrow), 0, err, 256) == OK, err.value
    assert open(out, "rb").read() == state
