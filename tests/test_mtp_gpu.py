"""The MTP drafting layer on the GPU (gcuda_set_mtp / gcuda_draft / gcuda_draft_next: Model::draft and
Model::draft_next, engine/src/model.cpp:1295-1480, over Model::forward_mtp, engine/src/model.cpp:4965-5039) against the
oracle's MTP pass (go_forward_mtp, pinned to the reference bit for bit in tests/test_oracle_mtp.py), on the MoE and
the dense model with the MTP layer:

- the prompt through the main model on the GPU, then the MTP pass over the prompt's positions in passes of up to 5
  rows, each fed the GPU's own hidden rows - the oracle is fed the same rows, so the MTP pass alone is compared: the
  last position's logits within max|d| <= 1e-2 x (max - min) of the oracle's, the draft the first maximum of the GPU's
  own logits (bit-exact), its probability softmax_at of those logits (rtol 1e-6: the double sum is grouped otherwise);
- the engine's loop: a verified batch's rows left on the device feed the next pass (hidden NULL);
- three chained drafts (gcuda_draft_next) from the pass's own output rows, each within the tolerance of the oracle's
  chain from its own;
- with a draft vocabulary (draft_vocab.bin, engine/src/model.cpp:803-827, 2135-2161): the pass multiplies only the
  draft head's rows - the ids inside the vocabulary, padded to whole tiles of 32 with copies of the first - so its
  logits are the oracle's full logits at those ids (each row's product stands alone) within the tolerance, the draft
  is the id at their first maximum and the probability softmax_at over the padded rows.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from geode_b200 import synth  # noqa: E402
import oracle_py as op  # noqa: E402

pytestmark = pytest.mark.gpu

TOL = 1e-2


def _close(got, ref, what):
    rr = float(ref.max() - ref.min())
    err = float(np.abs(got - ref).max())
    assert err <= TOL * rr, f"{what}: max|d| {err} vs range {rr}"


def _softmax_at(lg, best):
    d = (lg - lg[best]).astype(np.float32).astype(np.float64)
    return np.float32(1.0 / np.exp(d).sum())


def _check_draft(d, pr, lg, lg_ref, what):
    _close(lg, lg_ref, what)
    assert d == int(np.argmax(lg)), what   # (np.argmax: the first maximum, as std::max_element)
    assert np.isclose(pr, _softmax_at(lg, d), rtol=1e-6, atol=0), (what, pr, _softmax_at(lg, d))


@pytest.mark.parametrize("arch", ["qwen35moe", "qwen35"])
def test_mtp_drafts(arch, tmp_path):
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    from geode_b200.backend import Backend
    shape = synth.tiny_shape(arch, n_layers=4, ctx=640)
    d = str(tmp_path / "pack")
    synth.write_pack(d, shape, seed=61, mtp=True)
    ora = op.Oracle(d)
    st = ora.new_state(shape.ctx)
    be = Backend(d, context=shape.ctx, max_tokens=5)
    assert be.has_mtp
    rng = np.random.default_rng(62)
    V = shape.vocab
    L = 23
    prompt = rng.integers(0, V, L).astype(np.int32)
    hid = np.concatenate([be.verify(prompt[i:i + 5], logits=False, hidden=True)[1] for i in range(0, L, 5)])
    assert hid.shape == (L, shape.hidden)
    # the prompt's MTP positions 0 .. L - 2, passes of up to 5 rows, the GPU's hidden rows for both sides
    for p0 in range(0, L - 1, 5):
        p1 = min(p0 + 5, L - 1)
        dg, pr, lg = be.draft(prompt[p0 + 1:p1 + 1], p0, hidden=hid[p0:p1], logits=True)
        lg_ref, h_ref = ora.forward_mtp(st, prompt[p0 + 1:p1 + 1], hid[p0:p1], p0)
        _check_draft(dg, pr, lg, lg_ref, f"pass at {p0}")
    # a verified batch at L .. L + 4 (the draft and random tokens), its rows left on the device feed the MTP positions
    # L - 1 .. (the last prompt row first, from the host)
    dg, pr, lg = be.draft(np.array([dg], np.int32), L - 1, hidden=hid[L - 1:L], logits=True)
    lg_ref, h_ref = ora.forward_mtp(st, [dg], hid[L - 1:L], L - 1)
    batch = np.array([dg] + [int(t) for t in rng.integers(0, V, 4)], np.int32)
    _, hb = be.verify(batch, logits=False, hidden=True)
    nxt = np.array(list(batch[1:]) + [int(rng.integers(0, V))], np.int32)
    dg, pr, lg = be.draft(nxt, L, hidden=None, logits=True)
    lg_ref, h_ref = ora.forward_mtp(st, nxt, hb, L)
    _check_draft(dg, pr, lg, lg_ref, "pass on the device's rows")
    # chained drafts: the GPU from its own output rows, the oracle from its own
    q = L + 5
    tok = dg
    for i in range(3):
        dg, pr, lg = be.draft_next(tok, q, logits=True)
        lg_ref, h_ref = ora.forward_mtp(st, [tok], h_ref[None], q)
        _check_draft(dg, pr, lg, lg_ref, f"chained draft {i}")
        tok = dg
        q += 1
    be.close()


def test_mtp_refusals(tmp_path):
    """Drafting without an MTP layer, without verified rows, past the context or with a bad token: an error, and the
    handle still drafts afterwards."""
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    from geode_b200.backend import Backend, GcudaError
    shape = synth.tiny_shape("qwen35moe", n_layers=4, ctx=640)
    plain = str(tmp_path / "plain")
    synth.write_pack(plain, shape, seed=63)
    be = Backend(plain, context=shape.ctx, max_tokens=5)
    assert not be.has_mtp
    with pytest.raises(GcudaError):
        be.draft([1, 2], 0, hidden=np.zeros((2, shape.hidden), np.float32))
    be.close()
    d = str(tmp_path / "mtp")
    synth.write_pack(d, shape, seed=63, mtp=True)
    be = Backend(d, context=shape.ctx, max_tokens=5)
    H = shape.hidden
    with pytest.raises(GcudaError):
        be.draft([1, 2], 0)                                          # no verified batch to take the rows from
    with pytest.raises(GcudaError):
        be.draft_next(1, 0)                                          # no pass to chain from
    with pytest.raises(GcudaError):
        be.draft([1, shape.vocab], 0, hidden=np.zeros((2, H), np.float32))   # a token outside the vocabulary
    with pytest.raises(GcudaError):
        be.draft([1, 2], shape.ctx - 1, hidden=np.zeros((2, H), np.float32))  # past the context
    with pytest.raises(GcudaError):
        be.draft(list(range(6)), 0, hidden=np.zeros((6, H), np.float32))      # more rows than max_tokens
    dg, pr, _ = be.draft([1, 2], 0, hidden=np.ones((2, H), np.float32))
    assert 0 <= dg < shape.vocab and 0.0 < pr <= 1.0
    be.close()


@pytest.mark.parametrize("arch", ["qwen35moe", "qwen35"])
def test_mtp_draft_head(arch, tmp_path):
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    from geode_b200.backend import Backend, draft_vocab
    shape = synth.tiny_shape(arch, n_layers=4, ctx=640)
    d = str(tmp_path / "pack")
    synth.write_pack(d, shape, seed=71, mtp=True)
    V = shape.vocab
    rng = np.random.default_rng(72)
    raw_ids = list(rng.choice(V, 100, replace=False)) + [-1, V, V + 7]   # (the last three outside: left out)
    synth.write_draft_vocab(d, raw_ids)
    ids = draft_vocab(d, V)
    assert len(ids) == 128 and list(ids[:100]) == raw_ids[:100] and (ids[100:] == raw_ids[0]).all()
    ora = op.Oracle(d)
    st = ora.new_state(shape.ctx)
    be = Backend(d, context=shape.ctx, max_tokens=5)
    assert be.L.gcuda_draft_rows(be.g) == 128
    L = 13
    prompt = rng.integers(0, V, L).astype(np.int32)
    hid = np.concatenate([be.verify(prompt[i:i + 5], logits=False, hidden=True)[1] for i in range(0, L, 5)])

    def check(dg, pr, lg, lg_full, what):
        _close(lg, lg_full[ids], what)
        best = int(np.argmax(lg))
        assert dg == int(ids[best]), what
        assert np.isclose(pr, _softmax_at(lg, best), rtol=1e-6, atol=0), (what, pr, _softmax_at(lg, best))

    for p0 in range(0, L - 1, 5):
        p1 = min(p0 + 5, L - 1)
        dg, pr, lg = be.draft(prompt[p0 + 1:p1 + 1], p0, hidden=hid[p0:p1], logits=True)
        assert lg.shape == (128,)
        lg_ref, h_ref = ora.forward_mtp(st, prompt[p0 + 1:p1 + 1], hid[p0:p1], p0)
        check(dg, pr, lg, lg_ref, f"pass at {p0}")
    q, tok = L - 1, dg
    for i in range(2):
        dg, pr, lg = be.draft_next(tok, q, logits=True)
        lg_ref, h_ref = ora.forward_mtp(st, [tok], h_ref[None], q)
        check(dg, pr, lg, lg_ref, f"chained draft {i}")
        tok, q = dg, q + 1
    be.close()


def test_mtp_draft_after_keep(tmp_path):
    """The engine's loop drafts from the rows a step kept (ghost_draft(..., NULL) after verify_keep): after
    gcuda_keep(3) of a 5-row batch the device still holds rows 0..2, so a draft over 3 positions with hidden NULL
    runs, and equals the same draft fed those rows from the host bit for bit; 4 rows are refused."""
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    from geode_b200.backend import Backend, GcudaError
    shape = synth.tiny_shape("qwen35moe", n_layers=4, ctx=640)
    d = str(tmp_path / "pack")
    synth.write_pack(d, shape, seed=91, mtp=True)
    be = Backend(d, context=shape.ctx, max_tokens=5)
    rng = np.random.default_rng(92)
    toks = rng.integers(0, shape.vocab, 10).astype(np.int32)
    be.verify(toks[:5], logits=False)
    _, hid = be.verify(toks[5:10], logits=False, hidden=True)
    be.keep(3)
    nxt = np.array([toks[6], toks[7], int(rng.integers(0, shape.vocab))], np.int32)
    with pytest.raises(GcudaError):
        be.draft(np.append(nxt, 1), 5)
    d0, p0, lg0 = be.draft(nxt, 5, logits=True)
    d1, p1, lg1 = be.draft(nxt, 5, hidden=hid[:3], logits=True)
    assert (d0, np.float32(p0)) == (d1, np.float32(p1)) and np.array_equal(lg0, lg1)
    be.close()
