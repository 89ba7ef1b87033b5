"""The oracle against the reference engine at the benchmark configurations' own model shapes (where the reference build
is here): cfg 1 (one attention layer, hidden 2048, FFN 6144, vocab 32768, 1024 random KV positions), cfg 2 (the
24-layer dense hybrid, vocab 248320, 4096 random KV positions and random recurrent / conv states) and cfg 3 at full
width on 4 of its 40 layers (3 Gated DeltaNet : 1 attention, 256 experts top-8 with ff 512 and the shared expert,
vocab 248320, 8192 random KV positions - the whole model's pack is 20 GB). The starting state
goes into the reference through its own state file (written here by ghost_state_write, which the state-file tests pin
to the reference's save_state) and into the oracle directly; then 5 tokens through both: every logit equal. And the
acceptance rule at the full vocabulary, greedy and sampled."""
import ctypes as C
import os

import numpy as np
import pytest

from geode_b200 import synth
import oracle_py as op
from state_helpers import compact_kv as _compact_kv, random_state as _random_state
from test_state_file import HOST_SO, Shapes

pytestmark = pytest.mark.skipif(not op.have_reference(), reason="the reference build oracle/_ref is not here")


@pytest.mark.parametrize("cfg", [1, 2, 3])
def test_oracle_equals_reference_at_config_shape(cfg, tmp_path):
    shape = synth.baseline_shape(cfg)
    if cfg == 3:
        shape.n_layers = 4
        shape.layer_types = synth.hybrid_types(4)
    d = str(tmp_path / "pack")
    synth.write_pack(d, shape, seed=60 + cfg, fill="random")
    ora = op.Oracle(d)
    ctx = shape.ctx + 16
    st = ora.new_state(ctx)
    rng = np.random.default_rng(70 + cfg)
    _random_state(ora, st, shape.ctx - 8, rng)
    c = ora.cfg
    conv_dim = 2 * c.gdn_k_heads * c.gdn_k_dim + c.gdn_v_heads * c.gdn_v_dim
    s = Shapes(ora.n_attn, c.n_kv_heads, c.n_kv_heads * c.head_dim, c.hidden, c.n_layers,
               ora.n_gdn * conv_dim * max(0, c.conv_kernel - 1), ora.n_gdn * c.gdn_v_heads * c.gdn_k_dim * c.gdn_v_dim)
    H = C.CDLL(HOST_SO)
    H.ghost_state_fingerprint.restype = C.c_uint64
    H.ghost_state_fingerprint.argtypes = [C.c_char_p, C.POINTER(Shapes)]
    H.ghost_state_write.argtypes = [C.c_char_p, C.c_uint64, C.POINTER(Shapes), C.c_int32, C.c_int32, C.c_uint64,
                                    C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int32, C.c_char_p, C.c_size_t]
    kv, kvs = _compact_kv(ora, st)
    kv, kvs = np.ascontiguousarray(kv), np.ascontiguousarray(kvs)
    path = str(tmp_path / "start.state")
    err = C.create_string_buffer(256)
    fp = H.ghost_state_fingerprint(d.encode(), C.byref(s))
    assert H.ghost_state_write(path.encode(), fp, C.byref(s), st.pos, 0, 1, st.conv.ctypes.data, st.gdn.ctypes.data,
                               kv.ctypes.data, kvs.ctypes.data, 0, err, 256) == 0, err.value
    toks = rng.integers(0, shape.vocab, 5).astype(np.int32)
    ref = op.Reference(d, threads=os.cpu_count() or 1, ctx=ctx)
    try:
        ref.load_state(path)
        assert ref.pos == shape.ctx - 8
        want = ref.forward(toks, all_logits=True)["logits"]
    finally:
        ref.close()
    got = ora.forward(st, toks, logits=True)["logits"]
    assert np.array_equal(got, want)


@pytest.mark.parametrize("temperature,top_p,top_k", [(0.0, 1.0, 0), (0.7, 0.95, 20), (1.0, 1.0, 0)])
def test_accept_rule_full_vocab(temperature, top_p, top_k):
    """The acceptance rule (engine/src/geode.cpp:327-350 around geode::Sampler) at the full vocabulary, 248320: the
    oracle's kept count, next token and every row's sample equal the reference's, greedy and sampled, on rows of
    N(0, 3) logits whose drafts are planted (each row's greedy sample, then a wrong one) so that drafts stand and fall."""
    V = 248320
    rng = np.random.default_rng(int(temperature * 10) + top_k)
    R, O = op.reference_lib(), op.oracle_lib()
    for case in range(5):
        rows = (rng.standard_normal((5, V), dtype=np.float32) * 3).astype(np.float32)
        batch = np.zeros(5, np.int32)
        batch[0] = rng.integers(0, V)
        stand = case   # 0..4 greedy drafts planted (4: every draft stands, the bonus token is row 4's sample)
        for i in range(4):
            batch[i + 1] = int(np.argmax(rows[i])) if i < stand else int(rng.integers(0, V))
        seed = int(rng.integers(0, 2 ** 31))
        out = []
        for lib, fn in ((R, "ref_accept"), (O, "go_accept")):
            nxt = C.c_int(0)
            samples = np.zeros(5, np.int32)
            kept = getattr(lib, fn)(rows.ctypes.data, 5, V, batch.ctypes.data, temperature, top_p, top_k,
                                    C.c_uint64(seed), None, 0, C.byref(nxt), samples.ctypes.data)
            out.append((kept, nxt.value, samples.tolist()))
        assert out[0] == out[1], (case, out)


@pytest.mark.parametrize("temperature,top_p,top_k", [(0.0, 1.0, 0), (0.7, 0.95, 20)])
def test_accept_presence_full_vocab(temperature, top_p, top_k):
    """geode_generate's presence penalty (engine/src/geode.cpp:234-255) at the full vocabulary, 248320: the oracle's
    kept count, next token, samples and seen list after the step equal the reference's. The seen lists hold rows'
    maxima and 200 other ids; the drafts are the penalised greedy samples (every count 0..4 of them)."""
    V = 248320
    rng = np.random.default_rng(33 + top_k)
    R, O = op.reference_lib(), op.oracle_lib()
    for case in range(5):
        rows = (rng.standard_normal((5, V), dtype=np.float32) * 3).astype(np.float32)
        batch = rng.integers(0, V, 5).astype(np.int32)
        seen = [int(np.argmax(rows[i])) for i in range(4)] + [int(t) for t in rng.choice(V, 200, replace=False)]
        seen = list(dict.fromkeys(seen))
        op.plant_penalized_drafts(rows, batch, seen, 1.5, case)
        seed = int(rng.integers(0, 2 ** 31))
        a = op.accept_seen(R, rows, batch, temperature, top_p, top_k, seed, 1.5, seen, fn="ref_accept_seen")
        b = op.accept_seen(O, rows, batch, temperature, top_p, top_k, seed, 1.5, seen)
        assert a[:2] == b[:2] and np.array_equal(a[2], b[2]) and np.array_equal(a[3], b[3]), (case, a, b)
