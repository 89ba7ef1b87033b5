"""The C++ host side without a GPU (libgeode_host.so): its pack reader agrees with the manifest, and a broken pack is
an error with a message, not a crash."""
import ctypes as C
import json
import os

import numpy as np
import pytest

from geode_b200 import synth

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HOST_SO = os.path.join(ROOT, "geode_b200", "libgeode_host.so")


@pytest.fixture(scope="module")
def H():
    if not os.path.exists(HOST_SO):
        pytest.fail(f"{HOST_SO} is not built (python -m geode_b200.build)")
    L = C.CDLL(HOST_SO)
    L.ghost_pack_summary.argtypes = [C.c_char_p, C.c_char_p, C.c_size_t, C.c_char_p, C.c_size_t]
    return L


def _expected(d):
    m = json.load(open(os.path.join(d, "geode.json")))
    n = q4 = nbytes = 0
    for t in m["tensors"].values():
        count = int(np.prod(t["shape"]))
        n += 1
        if t["type"] == "q4":
            q4 += 1
            nbytes += t["shape"][0] * int(np.prod(t["shape"][1:])) // 16 * 9
        else:
            nbytes += count * (4 if t["type"] == "f32" else 2)
    c = m["config"]
    ebytes = sum(e["stride"] * c.get("num_experts", 0) for e in m.get("experts", {}).get("layers", []))
    return (f"arch={m['arch']} layers={c['num_hidden_layers']} hidden={c['hidden_size']} vocab={c['vocab_size']} "
            f"experts={c.get('num_experts', 0)} tensors={n} q4={q4} bytes={nbytes} expert_bytes={ebytes}")


@pytest.mark.parametrize("arch", ["qwen35moe", "qwen35"])
def test_pack_summary(H, tmp_path, arch):
    d = str(tmp_path)
    synth.write_pack(d, synth.tiny_shape(arch), seed=2)
    out, err = C.create_string_buffer(1024), C.create_string_buffer(1024)
    assert H.ghost_pack_summary(d.encode(), out, 1024, err, 1024) == 0, err.value
    assert out.value.decode() == _expected(d)


def test_broken_packs(H, tmp_path):
    out, err = C.create_string_buffer(512), C.create_string_buffer(512)
    assert H.ghost_pack_summary(str(tmp_path).encode(), out, 512, err, 512) != 0
    assert b"geode.json" in err.value
    d = str(tmp_path)
    synth.write_pack(d, synth.tiny_shape("qwen35moe"), seed=2)
    man = os.path.join(d, "geode.json")
    text = open(man).read()
    open(man, "w").write(text[: len(text) // 2])   # truncated manifest
    assert H.ghost_pack_summary(d.encode(), out, 512, err, 512) != 0
    assert b"geode.json" in err.value
    m = json.loads(text)
    name = next(iter(m["tensors"]))
    m["tensors"][name]["offset"] = 1 << 40   # past its file
    open(man, "w").write(json.dumps(m))
    assert H.ghost_pack_summary(d.encode(), out, 512, err, 512) != 0
    assert b"past its file" in err.value


def test_draft_vocab(tmp_path):
    """The draft vocabulary as the engine's GPU branch takes it (engine/src/model.cpp:2135-2161), which the Python
    binding and the C++ host both follow: the int32 ids inside the vocabulary in file order, padded to whole tiles of
    32 rows with copies of the first; no file, or no id inside the vocabulary: no draft head."""
    from geode_b200.backend import draft_vocab
    d = str(tmp_path)
    assert draft_vocab(d, 1024) is None
    synth.write_draft_vocab(d, [-5, 2000])
    assert draft_vocab(d, 1024) is None
    synth.write_draft_vocab(d, [7, -1, 1023, 1024, 3] + list(range(100, 130)))
    ids = draft_vocab(d, 1024)
    want = [7, 1023, 3] + list(range(100, 130))
    assert ids.dtype == np.int32 and len(ids) == 64
    assert list(ids[:len(want)]) == want and (ids[len(want):] == 7).all()
    synth.write_draft_vocab(d, list(range(64)))
    assert list(draft_vocab(d, 1024)) == list(range(64))
