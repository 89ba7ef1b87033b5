"""Single-token decode (the non-speculative step: Model::forward_batch with n = 1, engine/src/model.cpp:1095-1136 for
the engine's GPU path) through the verify backend - gcuda_verify with one token - against the oracle, on the MoE and
the dense model: every step's logits within max|d| <= 1e-2 x (max - min) of the oracle's, and the same tokens
verified as one batch on a second handle give rows within the same bound of the one-at-a-time logits."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from geode_b200 import synth  # noqa: E402
import oracle_py as op  # noqa: E402

pytestmark = pytest.mark.gpu

TOL = 1e-2


def _close(got, ref):
    span = ref.max(axis=-1) - ref.min(axis=-1)
    return np.abs(got - ref).max(axis=-1), span, bool(np.all(np.abs(got - ref).max(axis=-1) <= TOL * span))


@pytest.mark.parametrize("arch", ["qwen35moe", "qwen35"])
def test_decode_one_token_at_a_time(arch, tmp_path):
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    from geode_b200.backend import Backend
    shape = synth.tiny_shape(arch, n_layers=4, ctx=640)
    d = str(tmp_path / "pack")
    synth.write_pack(d, shape, seed=17)
    ora = op.Oracle(d)
    st = ora.new_state(shape.ctx)
    toks = np.random.default_rng(18).integers(0, shape.vocab, 5).astype(np.int32)
    one = Backend(d, context=64, max_tokens=5)
    batch = Backend(d, context=64, max_tokens=5)
    try:
        rows = []
        for t in toks:
            got, _ = one.verify(np.array([t], np.int32))
            ref = ora.forward(st, [t], logits=True)["logits"]
            err, span, ok = _close(got, ref)
            assert ok, f"token {t}: max|d| {err} vs range {span}"
            rows.append(got[0])
        assert one.pos == 5
        got_b, _ = batch.verify(toks)
        err, span, ok = _close(got_b, np.array(rows))
        assert ok, f"batched vs one at a time: max|d| {err} vs range {span}"
    finally:
        one.close()
        batch.close()
