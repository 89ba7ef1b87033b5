"""The acceptance microbench's configuration at full size: 256 sequences x 8 drafts, vocab 248320, target and draft
logits N(0, 3) in fp32, temperature 0.7, top-k 20, top-p 0.95, Philox seed 1234; greedy and rejection-sampling modes.

The drafts are the draft rows' argmax (a greedy drafter). Every 16th sequence's draft model agrees with the target
model on its first j rows (j = 0 .. 8 in turn), so accepted lengths from 0 to 8 occur; the other sequences' draft
rows are independent of the target's, as the configuration draws them.

- rejection sampling (gcuda_spec_reject, one launch over all 256 sequences): accepted lengths and next tokens equal
  the oracle's (go_spec_reject) for the planted sequences and a seeded sample of the others (the oracle sorts whole
  rows, ~50 ms a row, so not every sequence is re-run on the host; each sequence's result depends only on its rows);
- greedy (gcuda_op_greedy_verify): accepted lengths and next tokens equal the oracle's rule (go_accept at
  temperature 0) for every sequence.
"""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from geode_b200 import cuda_lib  # noqa: E402
import oracle_py as op  # noqa: E402

pytestmark = pytest.mark.gpu

S, K, V = 256, 8, 248320
T, TOP_P, TOP_K, SEED = 0.7, 0.95, 20, 1234
PLANT = 16


@pytest.fixture(scope="module")
def cfg5():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    gen = torch.Generator(device="cuda").manual_seed(5)
    target = torch.randn((S, K + 1, V), generator=gen, device="cuda") * 3
    draft = torch.randn((S, K, V), generator=gen, device="cuda") * 3
    for s in range(0, S, PLANT):
        j = (s // PLANT) % (K + 1)
        draft[s, :j] = target[s, :j]
    drafts = draft.argmax(dim=2).to(torch.int32).contiguous()
    torch.cuda.synchronize()
    yield target, draft, drafts
    del target, draft
    torch.cuda.empty_cache()


def test_cfg5_rejection_sampling(cfg5):
    from geode_b200.backend import GSampling, _sig
    target, draft, drafts = cfg5
    L = cuda_lib()
    _sig(L)
    O = op.oracle_lib()
    h_drafts = drafts.cpu().numpy()
    acc = np.zeros(S, np.int32)
    nxt = np.zeros(S, np.int32)
    err = C.create_string_buffer(256)
    g = L.gcuda_open(0, err, 256)
    assert g, err.value
    try:
        sp = GSampling(T, TOP_P, TOP_K)
        assert L.gcuda_spec_reject(g, target.data_ptr(), draft.data_ptr(), h_drafts.ctypes.data, S, K, V, C.byref(sp),
                                   SEED, acc.ctypes.data, nxt.ctypes.data) == 0
    finally:
        L.gcuda_close(g)
    rng = np.random.default_rng(1)
    others = [s for s in range(S) if s % PLANT]
    check = list(range(0, S, PLANT)) + sorted(rng.choice(others, 24, replace=False).tolist())
    for s in check:
        t = target[s].cpu().numpy()
        d = draft[s].cpu().numpy()
        n = C.c_int(0)
        ra = O.go_spec_reject(t.ctypes.data, d.ctypes.data, K, V, np.ascontiguousarray(h_drafts[s]).ctypes.data, T, TOP_P,
                              TOP_K, C.c_uint64(SEED), s, C.byref(n))
        assert (acc[s], nxt[s]) == (ra, n.value), s
    planted = acc[::PLANT]
    assert planted.tolist() == [(i % (K + 1)) for i in range(len(planted))]   # (q = p on the planted rows: all stand)
    assert (acc[[s for s in others]] == 0).mean() > 0.9   # independent draft models: nearly always the first falls


def test_cfg5_greedy(cfg5):
    target, draft, drafts = cfg5
    L = cuda_lib()
    O = op.oracle_lib()
    scratch = torch.empty(S * (K + 1), dtype=torch.int64, device="cuda")
    acc = torch.full((S,), -1, dtype=torch.int32, device="cuda")
    nxt = torch.full((S,), -1, dtype=torch.int32, device="cuda")
    assert L.gcuda_op_greedy_verify(target.data_ptr(), drafts.data_ptr(), S, K, V, scratch.data_ptr(), acc.data_ptr(),
                                    nxt.data_ptr(), None) == 0
    torch.cuda.synchronize()
    acc, nxt = acc.cpu().numpy(), nxt.cpu().numpy()
    h_drafts = drafts.cpu().numpy()
    for s in range(S):
        t = target[s].cpu().numpy()
        batch = np.concatenate([[0], h_drafts[s]]).astype(np.int32)
        n = C.c_int(0)
        kept = O.go_accept(t.ctypes.data, K + 1, V, batch.ctypes.data, 0.0, 1.0, 0, C.c_uint64(0), None, 0, C.byref(n),
                           np.zeros(K + 1, np.int32).ctypes.data)
        assert (acc[s], nxt[s]) == (kept - 1, n.value), s
    assert acc[::PLANT].tolist() == [(i % (K + 1)) for i in range(S // PLANT)]
