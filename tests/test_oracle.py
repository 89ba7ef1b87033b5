"""The oracle pinned: the C restatement (oracle/geode_oracle.c) against
  (a) the committed golden fixtures (tests/golden/, produced by the reference engine's own code, make_golden.py), and
  (b) the reference engine compiled from its sources (oracle/_ref), where that build exists (this container),
bit for bit. The restated q4 quantizer of the synthetic-pack writer (geode_b200/synth.py) is pinned the same way.
CPU only."""
import ctypes as C
import os

import numpy as np
import pytest

from geode_b200 import synth
import oracle_py as op

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden")
ref_only = pytest.mark.skipif(not op.have_reference(), reason="the reference build oracle/_ref is not here")


@pytest.fixture(scope="module")
def O():
    return op.oracle_lib()


@pytest.fixture(scope="module")
def R():
    return op.reference_lib() if op.have_reference() else None


def _golden(name):
    path = os.path.join(GOLDEN, name)
    if not os.path.exists(path):
        pytest.skip(f"golden fixture {name} missing")
    with np.load(path) as z:   # (materialized: an NpzFile member is a fresh array on every access)
        return {k: z[k] for k in z.files}


# ------------------------------------------------------------------------------------------- golden fixtures ----
def test_golden_kernels(O):
    g = _golden("kernels.npz")
    # E4M3 table
    tab = np.array([O.go_e4m3_value(b) for b in range(256)], np.float32)
    assert np.array_equal(tab.view(np.uint32)[np.isfinite(tab)], g["e4m3"].view(np.uint32)[np.isfinite(g["e4m3"])])
    # quantize_activation
    q, s, b = op.oracle_quantize_activation(O, g["act_x"])
    assert np.array_equal(q, g["act_q"]) and np.array_equal(s.view(np.uint32), g["act_scale"].view(np.uint32))
    assert np.array_equal(b, g["act_bsum"])
    # the int8 q4 GEMV
    y = op.oracle_matvec_q(O, g["w_packed"], int(g["w_rows"]), int(g["w_cols"]), float(g["w_global"]), g["w_x"])
    assert np.array_equal(y.view(np.uint32), g["w_y"].view(np.uint32))
    # the bf16 GEMV (8 partial sums)
    w, xs = g["bf_w"], g["bf_x"]
    ys = np.zeros((xs.shape[0], w.shape[0]), np.float32)
    O.go_matvec_bf16(w.ctypes.data, w.shape[0], w.shape[1], xs.shape[0], xs.ctypes.data, ys.ctypes.data)
    assert np.array_equal(ys.view(np.uint32), g["bf_y"].view(np.uint32))
    # route_topk
    for t in range(g["rt_logits"].shape[0]):
        ids, wt = op.oracle_route_topk(O, g["rt_logits"][t], int(g["rt_k"]))
        assert np.array_equal(ids, g["rt_ids"][t]) and np.array_equal(wt.view(np.uint32), g["rt_w"][t].view(np.uint32))
    # rmsnorm
    out = np.zeros_like(g["rn_x"])
    O.go_rmsnorm(g["rn_x"].ctypes.data, g["rn_w"].ctypes.data, out.ctypes.data, g["rn_x"].size, C.c_float(1e-6), 1)
    assert np.array_equal(out.view(np.uint32), g["rn_y"].view(np.uint32))
    # fast_exp
    fe = np.array([O.go_fast_exp(float(v)) for v in g["fe_x"]], np.float32)
    assert np.array_equal(fe.view(np.uint32), g["fe_y"].view(np.uint32))
    # the sampler's uniform stream
    u = op.oracle_uniforms(O, int(g["mt_seed"]), len(g["mt_u"]))
    assert np.array_equal(u.view(np.uint64), g["mt_u"].view(np.uint64))


def test_golden_q4_quantizer():
    g = _golden("kernels.npz")
    packed, s2 = synth.q4_quantize(g["qz_w"])
    assert np.array_equal(packed, g["qz_packed"]) and np.float32(s2) == np.float32(g["qz_s2"])


def test_golden_accept(O):
    g = _golden("accept.npz")
    rows, batch = g["rows"], g["batch"]
    for case in range(g["params"].shape[0]):
        T, P, K, seed = g["params"][case]
        nxt = C.c_int(0)
        samples = np.zeros(rows.shape[1], np.int32)
        kept = O.go_accept(rows[case].ctypes.data, rows.shape[1], rows.shape[2], batch[case].ctypes.data, float(T), float(P),
                           int(K), C.c_uint64(int(seed)), None, 0, C.byref(nxt), samples.ctypes.data)
        assert kept == g["kept"][case] and nxt.value == g["next"][case] and np.array_equal(samples, g["samples"][case])


def test_golden_accept_seen(O):
    """The acceptance with geode_generate's presence penalty (engine/src/geode.cpp:234-255) against the reference's
    outcomes: kept, next, every row's sample and the answer's seen list after the step, bit for bit."""
    g = _golden("accept_seen.npz")
    for case in range(g["params"].shape[0]):
        T, P, K, seed, pen = g["params"][case]
        seen = g["seen"][case][: g["n_seen"][case]]
        kept, nxt, samples, after = op.accept_seen(O, g["rows"][case], g["batch"][case], float(T), float(P), int(K),
                                                   int(seed), float(pen), seen)
        assert kept == g["kept"][case] and nxt == g["next"][case], case
        assert np.array_equal(samples, g["samples"][case]), case
        assert np.array_equal(after, g["seen_out"][case][: g["n_seen_out"][case]]), case


@pytest.mark.parametrize("name", ["model_moe", "model_dense"])
def test_golden_model(name):
    """The whole verify pass (forward_batch over a prompt, then 5 rows with every logit) on the committed tiny pack
    against the reference's logits and per-layer trace, bit for bit."""
    g = _golden(name + ".npz")
    import tempfile
    with tempfile.TemporaryDirectory() as d:
        shape = synth.tiny_shape("qwen35moe" if name == "model_moe" else "qwen35", n_layers=4, ctx=640)
        synth.write_pack(d, shape, seed=int(g["seed"]))
        ora = op.Oracle(d, attn_block=int(g["attn_block"]))
        st = ora.new_state(shape.ctx)
        o1 = ora.forward(st, g["prompt"], logits=True)
        assert np.array_equal(o1["logits"].view(np.uint32), g["prompt_logits"].view(np.uint32))
        o2 = ora.forward(st, g["toks"], logits=True, trace=True)
        assert np.array_equal(o2["logits"].view(np.uint32), g["logits"].view(np.uint32))
        for k in ("x", "mixer", "moe", "out"):
            assert np.array_equal(o2["trace"][k].view(np.uint32), g["trace_" + k].view(np.uint32)), k
        if name == "model_moe":
            assert np.array_equal(o2["trace"]["ids"], g["trace_ids"])


# ------------------------------------------------------------------------------------------- the live reference ----
@ref_only
def test_ref_q4_block(R):
    rng = np.random.default_rng(2)
    for trial in range(200):
        x = (rng.standard_normal(16) * rng.choice([1e-4, 0.02, 1.0])).astype(np.float32)
        if trial % 17 == 0:
            x[:] = 0
        s2 = np.float32(abs(rng.standard_normal()) * 0.01 + 1e-6)
        sb = C.c_uint8(0)
        codes = np.zeros(16, np.uint8)
        R.ref_q4_block(x.ctypes.data, C.c_float(s2), C.byref(sb), codes.ctypes.data)
        packed, _ = synth.q4_quantize(x.reshape(1, 16), s2)
        lo, hi = packed[0, :8] & 15, packed[0, :8] >> 4
        got = np.empty(16, np.uint8)
        got[0::2], got[1::2] = lo, hi
        assert packed[0, 8] == sb.value and np.array_equal(got, codes), trial


@ref_only
@pytest.mark.parametrize("arch", ["qwen35moe", "qwen35"])
def test_ref_model_bit_exact(tmp_path, arch):
    shape = synth.tiny_shape(arch, n_layers=4, ctx=640)
    synth.write_pack(str(tmp_path), shape, seed=3)
    ora = op.Oracle(str(tmp_path), attn_block=64)
    ref = op.Reference(str(tmp_path), threads=4, ctx=shape.ctx, attn_block=64)
    st = ora.new_state(shape.ctx)
    rng = np.random.default_rng(1)
    prompt = rng.integers(0, shape.vocab, 150)
    o1, r1 = ora.forward(st, prompt), ref.forward(prompt)
    assert np.array_equal(o1["logits"].view(np.uint32), r1["logits"].view(np.uint32))
    for _ in range(2):
        toks = rng.integers(0, shape.vocab, 5)
        o2, r2 = ora.forward(st, toks, trace=True), ref.forward(toks, trace=True)
        assert np.array_equal(o2["logits"].view(np.uint32), r2["logits"].view(np.uint32))
        for k in ("x", "mixer", "moe", "out", "ids", "weights"):
            assert np.array_equal(o2["trace"][k], r2["trace"][k]), k
    ref.close()


@ref_only
def test_ref_rollback(tmp_path):
    """The K=4 rollback the reference gives (save_state / load_state, then the kept prefix again) equals the oracle's
    state copy + prefix (engine/src/model.cpp:5-7: a batch gives the bits one token at a time gives)."""
    shape = synth.tiny_shape("qwen35moe", n_layers=4, ctx=640)
    synth.write_pack(str(tmp_path), shape, seed=4)
    ora = op.Oracle(str(tmp_path))
    ref = op.Reference(str(tmp_path), threads=2, ctx=shape.ctx)
    st = ora.new_state(shape.ctx)
    rng = np.random.default_rng(9)
    prompt = rng.integers(0, shape.vocab, 40)
    ora.forward(st, prompt, logits=False)
    ref.forward(prompt)
    path = str(tmp_path / "s.state")
    ref.save_state(path)
    before = st.copy()
    toks = rng.integers(0, shape.vocab, 5)
    ora.forward(st, toks)
    ref.forward(toks)
    kept = 2
    ref.load_state(path)
    ref.forward(toks[:kept])
    st = before
    ora.forward(st, toks[:kept], logits=False)
    nxt = rng.integers(0, shape.vocab, 5)
    a, b = ora.forward(st, nxt), ref.forward(nxt)
    assert np.array_equal(a["logits"].view(np.uint32), b["logits"].view(np.uint32))
    ref.close()


@ref_only
def test_ref_accept(R, O):
    rng = np.random.default_rng(6)
    V = 5000
    for case in range(12):
        rows = (rng.standard_normal((5, V)) * 3).astype(np.float32)
        batch = rng.integers(0, V, 5).astype(np.int32)
        # plant standing drafts: batch[i+1] = argmax row i for the first j rows
        j = case % 5
        for i in range(j):
            batch[i + 1] = int(np.argmax(rows[i]))
        T, P, K = [(0.0, 1.0, 0), (0.7, 0.95, 20), (0.7, 1.0, 0), (1.3, 0.8, 40)][case % 4]
        seed = int(rng.integers(0, 2 ** 40))
        n1, n2 = C.c_int(0), C.c_int(0)
        s1, s2 = np.zeros(5, np.int32), np.zeros(5, np.int32)
        k1 = R.ref_accept(rows.ctypes.data, 5, V, batch.ctypes.data, T, P, K, C.c_uint64(seed), None, 0, C.byref(n1),
                          s1.ctypes.data)
        k2 = O.go_accept(rows.ctypes.data, 5, V, batch.ctypes.data, T, P, K, C.c_uint64(seed), None, 0, C.byref(n2),
                         s2.ctypes.data)
        assert (k1, n1.value) == (k2, n2.value) and np.array_equal(s1, s2), case


@ref_only
def test_ref_accept_seen(R, O):
    """The presence penalty's acceptance, oracle against the live reference build: greedy and sampled, positive and
    negative penalties, seen lists holding rows' maxima, drafts planted as the penalised greedy samples."""
    rng = np.random.default_rng(16)
    V = 5000
    for case in range(16):
        rows = (rng.standard_normal((5, V)) * 3).astype(np.float32)
        batch = rng.integers(0, V, 5).astype(np.int32)
        seen = list(rng.choice(V, int(rng.integers(0, 40)), replace=False))
        for i in range(min(len(seen), 4)):
            seen[i] = int(np.argmax(rows[i]))
        seen = list(dict.fromkeys(int(t) for t in seen))
        pen = [2.0, -1.0, 0.5, 4.0][case % 4]
        op.plant_penalized_drafts(rows, batch, seen, pen, case % 5)
        T, P, K = [(0.0, 1.0, 0), (0.7, 0.95, 20), (0.0, 1.0, 0), (1.3, 0.8, 40)][case % 4]
        seed = int(rng.integers(0, 2 ** 40))
        a = op.accept_seen(R, rows, batch, T, P, K, seed, pen, seen, fn="ref_accept_seen")
        b = op.accept_seen(O, rows, batch, T, P, K, seed, pen, seen)
        assert a[:2] == b[:2] and np.array_equal(a[2], b[2]) and np.array_equal(a[3], b[3]), case


@ref_only
def test_ref_kernels(R, O):
    rng = np.random.default_rng(8)
    x = (rng.standard_normal(2048) * 2).astype(np.float32)
    q1, s1, b1 = np.zeros(2048, np.int8), np.zeros(128, np.float32), np.zeros(128, np.int32)
    R.ref_quantize_activation(x.ctypes.data, 2048, q1.ctypes.data, s1.ctypes.data, b1.ctypes.data)
    q2, s2, b2 = op.oracle_quantize_activation(O, x)
    assert np.array_equal(q1, q2) and np.array_equal(s1, s2) and np.array_equal(b1, b2)
    w, g = synth.q4_quantize((rng.standard_normal((64, 2048)) * 0.02).astype(np.float32))
    xs = rng.standard_normal((5, 2048)).astype(np.float32)
    y1 = np.zeros((5, 64), np.float32)
    R.ref_matvec_q(w.ctypes.data, 64, 2048, C.c_float(g), 6, 5, xs.ctypes.data, y1.ctypes.data)
    y2 = op.oracle_matvec_q(O, w, 64, 2048, g, xs)
    assert np.array_equal(y1.view(np.uint32), y2.view(np.uint32))
    for r in (0, 9, 63):
        d1 = np.zeros(2048, np.float32)
        R.ref_dequant_row(np.ascontiguousarray(w[r]).ctypes.data, 2048, C.c_float(g), 6, d1.ctypes.data)
        assert np.array_equal(d1.view(np.uint32), synth.q4_dequant(w[r:r + 1], 2048, g)[0].view(np.uint32))
    lg = (rng.standard_normal((20, 256)) * 2).astype(np.float32)
    for t in range(20):
        i1, w1 = np.zeros(8, np.int32), np.zeros(8, np.float32)
        R.ref_route_topk(lg[t].ctypes.data, 256, 8, i1.ctypes.data, w1.ctypes.data)
        i2, w2 = op.oracle_route_topk(O, lg[t], 8)
        assert np.array_equal(i1, i2) and np.array_equal(w1, w2)
    for v in np.concatenate([rng.standard_normal(100) * 30, [-100.0, 100.0, 0.0, -87.0, 88.0]]).astype(np.float32):
        assert np.float32(R.ref_fast_exp(float(v))).view(np.uint32) == np.float32(O.go_fast_exp(float(v))).view(np.uint32)
