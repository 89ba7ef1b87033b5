"""Parity at the benchmark's own model shape, BASELINE cfg 3 (the MoE 35B-A3B shape), at full width on 4 of its 40
layers (3 Gated DeltaNet : 1 attention; 256 experts top-8 with ff 512 and the shared expert; vocab 248320) from a
random 8192-position starting state - the subset tests/test_oracle_configs.py pins the oracle to the reference at,
bit for bit. The whole model's pack is 20 GB; its 40 layers are these 4 layers' kinds repeated.

Stage by stage, through gcuda_debug_trace (the reference's LayerTrace, engine/src/model.hpp:92-105):
- each layer's input x within 1e-2 x its row's range of the oracle's (x[0], the embedding rows, bit for bit);
- the routing in the step bit-exact given its logits: every layer's ids and weights equal route_topk
  (engine/src/model.cpp:4021-4065) run by the oracle on the step's own router logits, and the shared expert's gate
  equals sigmoid of its own gate logit (engine/src/model.cpp:4564-4567, glibc's expf) - bit for bit;
- the picks against the oracle's own picks (its router logits come from its own, slightly different, hidden rows):
  nearly all equal;
then the logits of the 5 rows within 1e-2 x range, greedy acceptance bit-exact on the GPU's logits (go_accept), and
after the rollback the next batch's logits within the tolerance again."""
import ctypes as C
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from geode_b200 import synth  # noqa: E402
import oracle_py as op  # noqa: E402
from state_helpers import compact_kv as _compact_kv, random_state as _random_state  # noqa: E402

pytestmark = pytest.mark.gpu

TOL = 1e-2


def _within(got, ref):
    rr = ref.max(axis=-1) - ref.min(axis=-1)
    err = np.abs(got - ref).max(axis=-1)
    return err, rr, bool(np.all(err <= TOL * rr))


def _sigmoid_glibc(x: np.ndarray) -> np.ndarray:
    libm = C.CDLL("libm.so.6")
    libm.expf.restype = C.c_float
    libm.expf.argtypes = [C.c_float]
    e = np.array([libm.expf(float(-v)) for v in x.ravel()], np.float32).reshape(x.shape)
    return (np.float32(1.0) / (np.float32(1.0) + e)).astype(np.float32)


@pytest.fixture(scope="module")
def cfg3(tmp_path_factory):
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    from geode_b200.backend import Backend
    shape = synth.baseline_shape(3)
    shape.n_layers = 4
    shape.layer_types = synth.hybrid_types(4)
    d = str(tmp_path_factory.mktemp("cfg3"))
    synth.write_pack(d, shape, seed=63, fill="random")
    ora = op.Oracle(d)
    ctx = shape.ctx + 16
    st = ora.new_state(ctx)
    rng = np.random.default_rng(73)
    _random_state(ora, st, shape.ctx - 8, rng)
    be = Backend(d, context=ctx, max_tokens=5)
    kv, kvs = _compact_kv(ora, st)
    be.state_put(st.conv, st.gdn, np.ascontiguousarray(kv), np.ascontiguousarray(kvs), st.pos)
    yield shape, ora, be, st, rng
    be.close()


def test_cfg3_layers_routes_logits_accept_rollback(cfg3):
    shape, ora, be, st, rng = cfg3
    O = op.oracle_lib()
    V, K = shape.vocab, shape.top_k
    pos0 = st.pos
    # the batch: the last accepted token, then two drafts the oracle's greedy model predicts (they stand), then two
    # random ones - so that acceptance stops partway and the rollback moves
    toks = [int(rng.integers(0, V))]
    s2 = st.copy()
    for _ in range(2):
        lg = ora.forward(s2, [toks[-1]], logits=True)["logits"][0]
        toks.append(int(np.argmax(lg)))
    toks += [int(t) for t in rng.integers(0, V, 2)]
    toks = np.array(toks, np.int32)
    before = st.copy()
    ref = ora.forward(st, toks, logits=True, trace=True)
    tr_ref = ref["trace"]

    # 1. the traced step (the logits stay on the device), then the same batch again from the same state for its logits
    conv, gdn = st.conv.copy(), st.gdn.copy()
    kv, kvs = _compact_kv(ora, before)
    kv, kvs = np.ascontiguousarray(kv), np.ascontiguousarray(kvs)
    tr = be.trace(toks)
    be.state_put(before.conv, before.gdn, kv, kvs, pos0)
    got, _ = be.verify(toks, logits=True)
    del conv, gdn

    # 2. each layer's input x
    assert np.array_equal(tr["x"][0].view(np.uint32), tr_ref["x"][0].view(np.uint32)), "the embedding rows"
    for l in range(shape.n_layers):
        err, rr, ok = _within(tr["x"][l], tr_ref["x"][l])
        assert ok, f"layer {l} input x: max|d| {err} vs range {rr}"
    err, rr, ok = _within(tr["x"][shape.n_layers], tr_ref["out"][shape.n_layers - 1])
    assert ok, f"the last layer's output: max|d| {err} vs range {rr}"

    # 3. the routing, bit-exact given the step's own router logits; the gate likewise
    same = total = 0
    for l in range(shape.n_layers):
        for t in range(len(toks)):
            row = tr["router_logits"][l, t]
            ids, w = op.oracle_route_topk(O, row[: shape.n_experts], K)
            assert np.array_equal(tr["ids"][l, t], ids), (l, t, tr["ids"][l, t], ids)
            assert np.array_equal(tr["weights"][l, t].view(np.uint32), w.view(np.uint32)), (l, t)
            gate = _sigmoid_glibc(row[shape.n_experts:])[0]
            assert np.float32(tr["gate"][l, t]).view(np.uint32) == gate.view(np.uint32), (l, t)
            same += len(set(tr["ids"][l, t].tolist()) & set(tr_ref["ids"][l, t].tolist()))
            total += K
        assert 1 <= tr["n_union"][l] <= len(toks) * K
    assert same >= 0.95 * total, f"picks equal to the oracle's: {same} of {total}"

    # 4. the logits, greedy acceptance on them, the rollback and the next batch
    err, rr, ok = _within(got, ref["logits"])
    assert ok, f"logits: max|d| {err} vs range {rr}"
    kept, nxt, samples = be.accept(0.0, 1.0, 0)
    rn = op.C.c_int(0)
    rs = np.zeros(5, np.int32)
    rk = O.go_accept(np.ascontiguousarray(got).ctypes.data, 5, V, toks.ctypes.data, 0.0, 1.0, 0, op.C.c_uint64(0),
                     None, 0, op.C.byref(rn), rs.ctypes.data)
    assert (kept, nxt) == (rk, rn.value) and np.array_equal(samples, rs)
    if kept < 5:
        be.keep(kept)
    st.__dict__.update(before.copy().__dict__)
    ora.forward(st, toks[:kept], logits=False)
    assert be.pos == st.pos
    toks2 = rng.integers(0, V, 5).astype(np.int32)
    ref2 = ora.forward(st, toks2, logits=True)["logits"]
    got2, _ = be.verify(toks2, logits=True)
    err, rr, ok = _within(got2, ref2)
    assert ok, f"after the rollback: max|d| {err} vs range {rr}"
