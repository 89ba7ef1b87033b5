"""GPU parity of the whole verify step (gcuda_verify / gcuda_keep / gcuda_accept) against the C oracle, itself pinned
bit for bit to the reference engine (tests/test_oracle.py).

- logits of the K+1 verified rows within max|d| <= 1e-2 x (max - min) of the oracle's row (fp32 accumulation; the GPU's
  exp / sin / cos and its attention order differ in the last bits, so the model is not bit-exact end to end);
- rollback: after keep(kept) the next batch's logits again within the tolerance (the Gated DeltaNet states restored
  as after token kept-1, the KV rows past it written over);
- acceptance: bit-exact given the same logits - the GPU's samples, kept and next equal the oracle's rule on the GPU's
  own logits, greedy and sampled (the reference's uniform stream, mt19937_64 -> generate_canonical).
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from geode_b200 import synth  # noqa: E402
import oracle_py as op  # noqa: E402
from state_helpers import compact_kv as _compact_kv  # noqa: E402

pytestmark = pytest.mark.gpu

TOL = 1e-2


def _shapes():
    tiny = synth.tiny_shape("qwen35moe", n_layers=4, ctx=640)
    heads = synth.ModelShape("heads-moe", "qwen35moe", 512, 4, 2048, synth.hybrid_types(4), n_heads=4, n_kv_heads=2,
                             head_dim=256, gdn_k_heads=2, gdn_v_heads=4, gdn_k_dim=128, gdn_v_dim=128, n_experts=32,
                             top_k=8, moe_ff=128, shared_ff=128, ctx=1100)
    # wide enough that the expert GEMVs take their streaming shapes (warp pairs on gate_up, one-tile units on down)
    wide = synth.ModelShape("wide-moe", "qwen35moe", 1024, 4, 4096, synth.hybrid_types(4), n_heads=4, n_kv_heads=2,
                            head_dim=256, gdn_k_heads=2, gdn_v_heads=4, gdn_k_dim=128, gdn_v_dim=128, n_experts=64,
                            top_k=8, moe_ff=256, shared_ff=256, ctx=1100)
    dense = synth.tiny_shape("qwen35", n_layers=4, ctx=640)
    return {"tiny-moe": tiny, "heads-moe": heads, "wide-moe": wide, "tiny-dense": dense}


SHAPES = _shapes()


@pytest.fixture(scope="module", params=list(SHAPES))
def setup(request, tmp_path_factory):
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    from geode_b200.backend import Backend
    shape = SHAPES[request.param]
    d = str(tmp_path_factory.mktemp(request.param))
    synth.write_pack(d, shape, seed=11)
    ora = op.Oracle(d)
    be = Backend(d, context=shape.ctx, max_tokens=5)
    rng = np.random.default_rng(5)
    st = ora.new_state(shape.ctx)
    prompt = rng.integers(0, shape.vocab, 300 if shape.ctx > 1000 else 120)
    ora.forward(st, prompt, logits=False)
    kv, kvs = _compact_kv(ora, st)
    be.state_put(st.conv, st.gdn, kv, kvs, st.pos)
    yield shape, ora, be, st, rng
    be.close()


def _close(got, ref):
    rng_ = ref.max(axis=-1) - ref.min(axis=-1)
    err = np.abs(got - ref).max(axis=-1)
    return err, rng_, bool(np.all(err <= TOL * rng_))


def test_verify_logits_and_rollback(setup):
    shape, ora, be, st, rng = setup
    for step in range(3):
        toks = rng.integers(0, shape.vocab, 5)
        before = st.copy()
        ref = ora.forward(st, toks, logits=True, hidden=True)
        got, hid = be.verify(toks, logits=True, hidden=True)
        err, rr, ok = _close(got, ref["logits"])
        assert ok, f"step {step}: max|d| {err} vs range {rr}"
        herr = np.abs(hid - ref["hidden"]).max()
        assert herr <= TOL * (np.abs(ref["hidden"]).max() + 1e-6), herr
        kept = int(rng.integers(1, 5))
        be.keep(kept)
        st.__dict__.update(before.copy().__dict__)
        ora.forward(st, toks[:kept], logits=False)
        assert be.pos == st.pos


def test_state_roundtrip(setup):
    """gcuda_state_get returns the state in the reference's layouts (the oracle's arrays): the KV rows, the conv and
    recurrent states - equal to the oracle's after the same batches (within the model tolerance for the floats)."""
    shape, ora, be, st, rng = setup
    conv, gdn = np.zeros_like(st.conv), np.zeros_like(st.gdn)
    kv_ref, kvs_ref = _compact_kv(ora, st)
    kv, kvs = np.zeros_like(kv_ref), np.zeros_like(kvs_ref)
    be.state_get(conv, gdn, kv, kvs, st.pos)
    assert np.allclose(conv, st.conv, rtol=1e-2, atol=1e-3)
    # the recurrent states per (layer, value head), normwise: a wrong index in one head moves that head's state by
    # about its own size; rounding-level differences carried through a few batches stay far below 1e-2
    c = ora.cfg
    if ora.n_gdn:
        a = gdn.reshape(ora.n_gdn, c.gdn_v_heads, -1).astype(np.float64)
        b = st.gdn.reshape(ora.n_gdn, c.gdn_v_heads, -1).astype(np.float64)
        rel = np.linalg.norm(a - b, axis=-1) / np.maximum(np.linalg.norm(b, axis=-1), 1e-30)
        assert rel.max() <= 1e-2, f"recurrent state per head: worst relative difference {rel.max():.2e}"
    # the int8 rows: equal, or one code apart where the GPU's float differs in the last bits before rounding - and
    # those rare
    d = np.abs(kv.astype(np.int32) - kv_ref.astype(np.int32))
    assert d.max() <= 1, f"KV codes {d.max()} apart"
    assert np.count_nonzero(d) <= 1e-2 * d.size, f"{np.count_nonzero(d)} of {d.size} KV codes differ"
    assert np.allclose(kvs, kvs_ref, rtol=1e-2, atol=1e-6)


def _planted(ora, st, t0, j, rng, vocab):
    """t0, then j drafts that the (greedy) model itself predicts, then random ones: a batch where the first j drafts
    stand (engine/src/geode.cpp:327-350), so partial acceptance and rollback really happen."""
    s2 = st.copy()
    toks = [int(t0)]
    for i in range(4):
        if i < j:
            lg = ora.forward(s2, [toks[-1]], logits=True)["logits"][0]
            toks.append(int(np.argmax(lg)))
        else:
            toks.append(int(rng.integers(0, vocab)))
    return np.array(toks, dtype=np.int32)


@pytest.mark.parametrize("temperature,top_p,top_k", [(0.0, 1.0, 0), (0.7, 0.95, 20), (0.7, 1.0, 0), (1.3, 0.8, 0)])
def test_accept_bit_exact(setup, temperature, top_p, top_k):
    shape, ora, be, st, rng = setup
    O = op.oracle_lib()
    for rep in range(3):
        j = int(rng.integers(0, 5))
        toks = _planted(ora, st, rng.integers(0, shape.vocab), j, rng, shape.vocab)
        before = st.copy()
        got, _ = be.verify(toks, logits=True)
        seed = int(rng.integers(0, 2 ** 31))
        u = op.oracle_uniforms(O, seed, 5)
        kept, nxt, samples = be.accept(temperature, top_p, top_k, uniforms=u)
        ref_samples = np.zeros(5, np.int32)
        ref_next = op.C.c_int(0)
        ref_kept = O.go_accept(got.ctypes.data, 5, shape.vocab, toks.ctypes.data, temperature, top_p, top_k,
                               op.C.c_uint64(seed), None, 0, op.C.byref(ref_next), ref_samples.ctypes.data)
        assert kept == ref_kept and nxt == ref_next.value and np.array_equal(samples, ref_samples), \
            (kept, ref_kept, nxt, ref_next.value, samples, ref_samples)
        if temperature == 0.0:
            assert kept >= min(5, j + 1) - (1 if j else 0)   # the planted drafts (nearly always) stand
        if kept < 5:
            be.keep(kept)
        st.__dict__.update(before.copy().__dict__)
        ora.forward(st, toks[:kept], logits=False)
        assert be.pos == st.pos


@pytest.mark.parametrize("temperature,top_p,top_k,penalty", [(0.0, 1.0, 0, 2.0), (0.0, 1.0, 0, -1.0),
                                                              (0.7, 0.95, 20, 1.5), (1.0, 1.0, 0, 0.75)])
def test_accept_presence_penalty(setup, temperature, top_p, top_k, penalty):
    """gcuda_accept with geode_generate's presence penalty (engine/src/geode.cpp:234-255): the seen list holds the
    oracle's greedy maxima of the batch's rows and random ids, the drafts are the oracle's penalised greedy samples;
    the GPU's kept, next and samples equal the oracle's rule (go_accept_seen, pinned to the reference) on the GPU's own
    logits bit for bit, and the penalty is seen to move a greedy sample. Between the reps the handle's rejection
    sampler reallocates its scratch, which must leave the accept's device copy of the seen list alone."""
    shape, ora, be, st, rng = setup
    O = op.oracle_lib()
    V = shape.vocab
    moved = False
    for rep in range(3):
        t0 = int(rng.integers(0, V))
        lg = ora.forward(st.copy(), [t0] + [int(t) for t in rng.integers(0, V, 4)], logits=True)["logits"]
        seen = list(dict.fromkeys([int(np.argmax(lg[i])) for i in range(2)] +
                                  [int(t) for t in rng.choice(V, 30, replace=False)]))
        toks = np.array([t0, 0, 0, 0, 0], np.int32)
        toks[1:] = rng.integers(0, V, 4)
        op.plant_penalized_drafts(lg, toks, seen, penalty, int(rng.integers(0, 5)))
        before = st.copy()
        got, _ = be.verify(toks, logits=True)
        seed = int(rng.integers(0, 2 ** 31))
        u = op.oracle_uniforms(O, seed, 5)
        kept, nxt, samples = be.accept(temperature, top_p, top_k, uniforms=u, presence_penalty=penalty, seen=seen)
        ref_kept, ref_next, ref_samples, _ = op.accept_seen(O, got, toks, temperature, top_p, top_k, seed, penalty,
                                                            seen)
        assert kept == ref_kept and nxt == ref_next and np.array_equal(samples, ref_samples), \
            (kept, ref_kept, nxt, ref_next, samples, ref_samples)
        # the handle's rejection sampler grows its own scratch here (S rises every rep); the accept's seen list on the
        # device must outlive that - the next rep's list is no longer, so its buffer is reused
        from geode_b200.backend import GSampling
        S = 2 + 3 * rep
        tgt = torch.from_numpy(np.ascontiguousarray(np.tile(got[None], (S, 1, 1)))).cuda()
        dft = torch.from_numpy(np.ascontiguousarray(np.tile(got[None, :4], (S, 1, 1)))).cuda()
        dd = np.ascontiguousarray(np.tile(toks[1:], S).astype(np.int32))
        acc, nx = np.zeros(S, np.int32), np.zeros(S, np.int32)
        assert be.L.gcuda_spec_reject(be.g, tgt.data_ptr(), dft.data_ptr(), dd.ctypes.data, S, 4, V,
                                      op.C.byref(GSampling(0.7, 1.0, 0)), 5, acc.ctypes.data, nx.ctypes.data) == 0
        if temperature == 0.0:
            moved |= any(samples[i] != int(np.argmax(got[i])) for i in range(kept))
        if kept < 5:
            be.keep(kept)
        st.__dict__.update(before.copy().__dict__)
        ora.forward(st, toks[:kept], logits=False)
        assert be.pos == st.pos
    if temperature == 0.0 and penalty > 0:
        assert moved, "the penalty never changed a greedy sample: the test does not exercise it"


@pytest.mark.parametrize("mode", ["greedy", "reject"])
def test_device_loop_step(setup, mode):
    """The device-resident step (gcuda_step_device: graph, greedy acceptance, decision, rollback on the device; and
    gcuda_step_device_reject with rejection sampling): its kept count equals the oracle's rule on the logits the same
    batch gives from the same state (gcuda_verify, then the state put back), and after its rollback the next batch's
    logits still match the oracle's."""
    shape, ora, be, st, rng = setup
    O = op.oracle_lib()
    V = shape.vocab
    for rep in range(3):
        j = int(rng.integers(0, 5))
        toks = _planted(ora, st, rng.integers(0, V), j, rng, V)
        before = st.copy()
        pos0 = be.pos
        conv, gdn = np.zeros_like(st.conv), np.zeros_like(st.gdn)
        kv, kvs = _compact_kv(ora, st)
        kv, kvs = np.zeros_like(kv), np.zeros_like(kvs)
        be.state_get(conv, gdn, kv, kvs, pos0)
        got, _ = be.verify(toks, logits=True)
        be.state_put(conv, gdn, kv, kvs, pos0)
        be.begin_device_loop(toks)
        if mode == "greedy":
            be.step_device(5)
            nxt = op.C.c_int(0)
            ref_kept = O.go_accept(got.ctypes.data, 5, V, toks.ctypes.data, 0.0, 1.0, 0, op.C.c_uint64(0), None, 0,
                                   op.C.byref(nxt), np.zeros(5, np.int32).ctypes.data)
        else:
            draft = np.ascontiguousarray(got[:4] + (rng.standard_normal((4, V)) * 0.3).astype(np.float32))
            d_draft = torch.from_numpy(draft).cuda()
            seed = 4242
            be.step_device_reject(5, d_draft.data_ptr(), 0.7, 0.95, 20, seed=seed)
            key = (seed + 0x9E3779B97F4A7C15 * rep) & (2 ** 64 - 1)   # (the handle's rep-th such step)
            nxt = op.C.c_int(0)
            acc = O.go_spec_reject(got.ctypes.data, draft.ctypes.data, 4, V, np.ascontiguousarray(toks[1:]).ctypes.data,
                                   0.7, 0.95, 20, op.C.c_uint64(key), 0, op.C.byref(nxt))
            ref_kept = acc + 1
        steps, _, kept = be.sync_step()
        assert steps == 1 and kept == ref_kept, (mode, rep, kept, ref_kept)
        assert be.pos == pos0 + kept
        st.__dict__.update(before.copy().__dict__)
        ora.forward(st, toks[:kept], logits=False)
    toks = rng.integers(0, V, 5)
    ref = ora.forward(st, toks, logits=True)
    got, _ = be.verify(toks, logits=True)
    err, rr, ok = _close(got, ref["logits"])
    assert ok, f"after the device steps: max|d| {err} vs range {rr}"
