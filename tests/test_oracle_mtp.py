"""The MTP drafting layer's oracle (go_forward_mtp: Model::forward_mtp, engine/src/model.cpp:4965-5039), pinned to the
reference engine bit for bit - the next row after the verify step: the layer that makes the drafts.

- against the golden fixtures tests/golden/mtp_moe.npz and mtp_dense.npz (made by the reference build,
  tests/golden/make_golden.py): on the tiny pack written again from their seed, the main model's hidden rows after a
  prompt, the MTP pass over the prompt's positions (the last position's logits and its output after mtp.norm), and one
  chained position fed its own draft, every float equal;
- against the live reference build where it exists (oracle/_ref), on another seed;
- a pack with the MTP layer is the pack without it plus the layer's tensors: every other tensor the same bytes.
"""
import json
import os

import numpy as np
import pytest

from geode_b200 import synth
import oracle_py as op

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
ref_only = pytest.mark.skipif(not op.have_reference(), reason="the reference build oracle/_ref is not here")


def _oracle_run(d, prompt, ctx=640):
    ora = op.Oracle(d)
    st = ora.new_state(ctx)
    hid = ora.forward(st, prompt, logits=False, hidden=True)["hidden"]
    lg1, h1 = ora.forward_mtp(st, prompt[1:], hid[:-1], 0)
    draft = int(np.argmax(lg1))
    lg2, h2 = ora.forward_mtp(st, [draft], h1[None], len(prompt) - 1)
    return hid, lg1, h1, draft, lg2, h2


@pytest.mark.parametrize("arch,name", [("qwen35moe", "mtp_moe"), ("qwen35", "mtp_dense")])
def test_mtp_golden(arch, name, tmp_path):
    g = np.load(os.path.join(GOLDEN, name + ".npz"))
    shape = synth.tiny_shape(arch, n_layers=4, ctx=640)
    d = str(tmp_path / "pack")
    synth.write_pack(d, shape, seed=int(g["seed"]), mtp=True)
    hid, lg1, h1, draft, lg2, h2 = _oracle_run(d, g["prompt"])
    assert np.array_equal(hid, g["hidden"])
    assert np.array_equal(lg1, g["logits1"]) and np.array_equal(h1, g["mtp_hidden1"])
    assert draft == int(g["draft"])
    assert np.array_equal(lg2, g["logits2"]) and np.array_equal(h2, g["mtp_hidden2"])


@ref_only
@pytest.mark.parametrize("arch", ["qwen35moe", "qwen35"])
def test_mtp_live_reference(arch, tmp_path):
    shape = synth.tiny_shape(arch, n_layers=4, ctx=640)
    d = str(tmp_path / "pack")
    synth.write_pack(d, shape, seed=57, mtp=True)
    prompt = np.random.default_rng(58).integers(0, shape.vocab, 33).astype(np.int32)
    ref = op.Reference(d, ctx=shape.ctx, draft=True)
    try:
        ref.forward(prompt, all_logits=False)
        hid_r = ref.hidden_rows(len(prompt))
        lg1_r, h1_r = ref.mtp(prompt[1:], hid_r[:-1], 0)
        draft_r = int(np.argmax(lg1_r))
        lg2_r, h2_r = ref.mtp([draft_r], h1_r[None], len(prompt) - 1)
    finally:
        ref.close()
    hid, lg1, h1, draft, lg2, h2 = _oracle_run(d, prompt)
    assert np.array_equal(hid, hid_r)
    assert np.array_equal(lg1, lg1_r) and np.array_equal(h1, h1_r) and draft == draft_r
    assert np.array_equal(lg2, lg2_r) and np.array_equal(h2, h2_r)


def test_mtp_pack_is_the_pack_plus_the_layer(tmp_path):
    shape = synth.tiny_shape("qwen35moe", n_layers=4, ctx=640)
    a, b = str(tmp_path / "a"), str(tmp_path / "b")
    synth.write_pack(a, shape, seed=9)
    synth.write_pack(b, shape, seed=9, mtp=True)
    ma, mb = (json.load(open(os.path.join(x, "geode.json"))) for x in (a, b))
    assert "mtp" not in ma and mb["mtp"]["experts"]["stride"] == ma["experts"]["layers"][0]["stride"]
    assert {k: v for k, v in mb["tensors"].items() if not k.startswith("mtp.")} == ma["tensors"]
    for f in ("dense.bin", "experts.bin"):
        fa, fb = (open(os.path.join(x, f), "rb").read() for x in (a, b))
        assert fb[:len(fa)] == fa and len(fb) > len(fa)
