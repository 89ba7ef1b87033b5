"""GPU parity of the operator layer (include/geode_cuda.h gcuda_op_*) against the C oracle, which itself is pinned
bit for bit to the reference engine (tests/test_oracle.py). Every check here is bit-exact: the q4 GEMV, the
activation quantizer, dequantized weights, the bf16 router GEMV and route_topk all reproduce the reference's
integer and float operation order."""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from geode_b200 import cuda_lib, synth  # noqa: E402
import oracle_py as op  # noqa: E402

pytestmark = pytest.mark.gpu


def _dev(a: np.ndarray):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _p(t) -> int:
    return t.data_ptr()


@pytest.fixture(scope="module")
def L():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    return cuda_lib()


@pytest.fixture(scope="module")
def O():
    return op.oracle_lib()


def _tiles(L, packed, rows, cols):
    d_pack = _dev(packed)
    tb = L.gcuda_op_q4_tiled_bytes(rows, cols)
    d_t = torch.zeros(tb, dtype=torch.uint8, device="cuda")
    assert L.gcuda_op_q4_relayout(_p(d_pack), rows, cols, _p(d_t), None) == 0
    return d_t


def _quant(L, x):
    n, cols = x.shape
    d_x = _dev(x.astype(np.float32))
    q = torch.zeros((n, cols), dtype=torch.int8, device="cuda")
    s = torch.zeros((n, cols // 16), dtype=torch.float32, device="cuda")
    b = torch.zeros((n, cols // 16), dtype=torch.int32, device="cuda")
    assert L.gcuda_op_quantize(_p(d_x), n, cols, _p(q), _p(s), _p(b), None) == 0
    return q, s, b


@pytest.mark.parametrize("cols", [512, 2048, 4096])
def test_quantize_bit_exact(L, O, cols):
    rng = np.random.default_rng(cols)
    x = rng.standard_normal((5, cols)).astype(np.float32) * 3
    x[0, :16] = 0.0  # an all-zero block: scale 0, codes 0
    q, s, b = _quant(L, x)
    torch.cuda.synchronize()
    for t in range(5):
        rq, rs, rb = op.oracle_quantize_activation(O, x[t])
        assert np.array_equal(q[t].cpu().numpy(), rq)
        assert np.array_equal(s[t].cpu().numpy().view(np.uint32), rs.view(np.uint32))
        assert np.array_equal(b[t].cpu().numpy(), rb)


@pytest.mark.parametrize("H", [256, 2048, 4096])
def test_norm_quant_bit_exact(L, O, H):
    """The step's norm-and-quantize kernel (k_norm_quant, without the MoE combine) against rmsnorm with the
    zero-centred weight (engine/src/kernels.cpp:1520-1529) then quantize_activation (engine/src/kernels.cpp:1254-1295)
    in the oracle, pinned to the reference: hf, codes, scales and block sums bit for bit. The kernel sums the squares
    in double in another order than the reference's sequential loop; every product is exact in double, and the float
    of the mean square matched on every row of these tests."""
    rng = np.random.default_rng(H)
    n = 8
    x = (rng.standard_normal((n, H)) * rng.uniform(0.1, 30.0, (n, 1))).astype(np.float32)
    x[1, :16] = 0.0   # a zero block after the norm: scale 0, codes 0
    w = (rng.standard_normal(H) * 0.1).astype(np.float32)
    eps = 1e-6
    d_x, d_w = _dev(x), _dev(w)
    hf = torch.zeros((n, H), dtype=torch.float32, device="cuda")
    q = torch.zeros((n, H), dtype=torch.int8, device="cuda")
    sc = torch.zeros((n, H // 16), dtype=torch.float32, device="cuda")
    bs = torch.zeros((n, H // 16), dtype=torch.int32, device="cuda")
    assert L.gcuda_op_norm_quant(_p(d_x), n, H, _p(d_w), eps, _p(hf), _p(q), _p(sc), _p(bs), None) == 0
    torch.cuda.synchronize()
    for t in range(n):
        ref = np.zeros(H, np.float32)
        O.go_rmsnorm(x[t].ctypes.data, w.ctypes.data, ref.ctypes.data, H, eps, 1)
        assert np.array_equal(hf[t].cpu().numpy().view(np.uint32), ref.view(np.uint32)), t
        rq, rs, rb = op.oracle_quantize_activation(O, ref)
        assert np.array_equal(q[t].cpu().numpy(), rq), t
        assert np.array_equal(sc[t].cpu().numpy().view(np.uint32), rs.view(np.uint32)), t
        assert np.array_equal(bs[t].cpu().numpy(), rb), t


@pytest.mark.parametrize("rows,cols,n", [(64, 512, 1), (1024, 2048, 5), (96, 4096, 3), (256, 2048, 8)])
def test_q4_gemv_bit_exact(L, O, rows, cols, n):
    rng = np.random.default_rng(rows + cols + n)
    w = rng.standard_normal((rows, cols)).astype(np.float32) * 0.02
    packed, g = synth.q4_quantize(w)
    d_t = _tiles(L, packed, rows, cols)
    x = rng.standard_normal((n, cols)).astype(np.float32)
    q, s, b = _quant(L, x)
    y = torch.zeros((n, rows), dtype=torch.float32, device="cuda")
    assert L.gcuda_op_q4_gemv(_p(d_t), rows, cols, g, _p(q), _p(s), _p(b), n, _p(y), None) == 0
    torch.cuda.synchronize()
    ref = op.oracle_matvec_q(O, packed, rows, cols, g, x)
    got = y.cpu().numpy()
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), np.abs(got - ref).max()


def test_q4_dequant_bit_exact(L):
    rng = np.random.default_rng(7)
    rows, cols = 96, 2048
    packed, g = synth.q4_quantize(rng.standard_normal((rows, cols)).astype(np.float32) * 0.02)
    d_t = _tiles(L, packed, rows, cols)
    sel = np.array([0, 5, 17, 63, 95], dtype=np.int64)
    out = torch.zeros((len(sel), cols), dtype=torch.float32, device="cuda")
    assert L.gcuda_op_q4_dequant(_p(d_t), cols, g, _p(_dev(sel)), len(sel), _p(out), None) == 0
    torch.cuda.synchronize()
    ref = synth.q4_dequant(packed[sel], cols, g)
    assert np.array_equal(out.cpu().numpy().view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("rows,n", [(257, 5), (16, 2)])
def test_bf16_gemv_bit_exact(L, O, rows, n):
    rng = np.random.default_rng(rows)
    cols = 2048
    w = synth.bf16_bits(rng.standard_normal((rows, cols)).astype(np.float32) * 0.05)
    x = rng.standard_normal((n, cols)).astype(np.float32)
    y = torch.zeros((n, rows), dtype=torch.float32, device="cuda")
    assert L.gcuda_op_bf16_gemv(_p(_dev(w)), rows, cols, _p(_dev(x)), n, _p(y), None) == 0
    torch.cuda.synchronize()
    ref = np.zeros((n, rows), np.float32)
    O.go_matvec_bf16(w.ctypes.data, rows, cols, n, x.ctypes.data, ref.ctypes.data)
    assert np.array_equal(y.cpu().numpy().view(np.uint32), ref.view(np.uint32))


def test_route_topk_bit_exact(L, O):
    rng = np.random.default_rng(3)
    n, E, K = 64, 256, 8
    lg = (rng.standard_normal((n, E)) * 2).astype(np.float32)
    lg[1, 10] = lg[1, 20] = lg[1].max() + 1  # an exact tie: the lower index first
    ids = torch.zeros((n, K), dtype=torch.int32, device="cuda")
    w = torch.zeros((n, K), dtype=torch.float32, device="cuda")
    assert L.gcuda_op_route_topk(_p(_dev(lg)), n, E, K, _p(ids), _p(w), None) == 0
    torch.cuda.synchronize()
    for t in range(n):
        rid, rw = op.oracle_route_topk(O, lg[t], K)
        assert np.array_equal(ids[t].cpu().numpy(), rid)
        assert np.array_equal(w[t].cpu().numpy().view(np.uint32), rw.view(np.uint32))


@pytest.mark.parametrize("n,E,K", [(5, 256, 8), (8, 128, 8), (1, 64, 4), (3, 1024, 8)])
def test_route_union_bit_exact(L, O, n, E, K):
    """The in-step routing kernel: each token's picks and weights bit-exact against route_topk, exact ties going to the
    lower id; the union ascending with every pick's slot and token mask; the shared expert's gate."""
    rng = np.random.default_rng(E + n)
    lg = (rng.standard_normal((n, E + 1)) * 2).astype(np.float32)
    lg[0, 5] = lg[0, 9] = lg[0, 40] = lg[0, :E].max() + 0.5   # a three-way tie at the top
    if n > 1:
        lg[1, :E] = lg[0, :E]                                  # two tokens with the same picks
    if n > 2:
        lg[2, 3:E] = -200.0                                    # 3 non-zero probabilities: K - 3 picks tie at 0
    size = L.gcuda_op_route_out_bytes()
    out = torch.zeros(size, dtype=torch.uint8, device="cuda")
    assert L.gcuda_op_route_union(_p(_dev(lg)), n, E, K, _p(out), size, None) == 0
    torch.cuda.synchronize()
    raw = out.cpu().numpy().view(np.int32)
    nu, ex, mask = raw[0], raw[1:65], raw[65:129]
    slot = raw[129:129 + 512].reshape(64, 8)
    ids = raw[641:705][:n * K].reshape(n, K)
    w = raw[705:769].view(np.float32)[:n * K].reshape(n, K)
    gs = raw[769:777].view(np.float32)[:n]
    picks = []
    for t in range(n):
        rid, rw = op.oracle_route_topk(O, np.ascontiguousarray(lg[t, :E]), K)
        assert np.array_equal(ids[t], rid), t
        assert np.array_equal(w[t].view(np.uint32), rw.view(np.uint32)), t
        picks.append(list(rid))
        x = np.float32(lg[t, E])
        ref_gs = np.float32(1.0) / (np.float32(1.0) + np.float32(np.exp(-np.float64(x))))
        assert gs[t].view(np.uint32) == np.float32(ref_gs).view(np.uint32)
    union = sorted({int(e) for p in picks for e in p})
    assert nu == len(union) and list(ex[:nu]) == union
    for u, e in enumerate(union):
        m = 0
        for t in range(n):
            if e in picks[t]:
                m |= 1 << t
                assert slot[u, t] == t * K + picks[t].index(e)
        assert mask[u] == m


@pytest.mark.parametrize("temperature,top_p,top_k", [(0.7, 0.95, 20), (1.0, 1.0, 0), (0.5, 0.8, 64)])
def test_spec_reject_bit_exact(L, O, temperature, top_p, top_k):
    """Rejection sampling (not in the reference; the oracle restates Leviathan et al.'s algorithm): accepted lengths
    and next tokens equal the oracle's for every sequence, with Philox uniforms keyed by (seed, sequence, row)."""
    from geode_b200.backend import GSampling, _sig
    _sig(L)
    rng = np.random.default_rng(int(temperature * 100) + top_k)
    S, k, V = 12, 4, 4096
    target = (rng.standard_normal((S, k + 1, V)) * 3).astype(np.float32)
    draft = target[:, :k, :] + (rng.standard_normal((S, k, V)) * 0.3).astype(np.float32)   # a close draft model
    drafts = np.zeros((S, k), np.int32)
    for s_ in range(S):   # drafts from the draft rows' argmax, some replaced at random
        drafts[s_] = np.argmax(draft[s_], axis=1)
        if s_ % 3 == 1:
            drafts[s_, s_ % k] = rng.integers(0, V)
    err = C.create_string_buffer(256)
    g = L.gcuda_open(0, err, 256)
    assert g, err.value
    try:
        d_t, d_d = _dev(target), _dev(np.ascontiguousarray(draft))
        acc = np.zeros(S, np.int32)
        nxt = np.zeros(S, np.int32)
        sp = GSampling(temperature, top_p, top_k)
        assert L.gcuda_spec_reject(g, _p(d_t), _p(d_d), drafts.ctypes.data, S, k, V, C.byref(sp), 1234,
                                   acc.ctypes.data, nxt.ctypes.data) == 0
    finally:
        L.gcuda_close(g)
    for s_ in range(S):
        n = C.c_int(0)
        ra = O.go_spec_reject(np.ascontiguousarray(target[s_]).ctypes.data, np.ascontiguousarray(draft[s_]).ctypes.data, k, V,
                              np.ascontiguousarray(drafts[s_]).ctypes.data, temperature, top_p, top_k, 1234, s_, C.byref(n))
        assert (acc[s_], nxt[s_]) == (ra, n.value), s_
    assert len(set(acc.tolist())) > 1   # (sequences stop at different drafts)


@pytest.mark.parametrize("V,offset", [(4096, 0), (1001, 0), (4096, 1)])
def test_greedy_verify_bit_exact(L, O, V, offset):
    """gcuda_op_greedy_verify (k_argmax_rows + k_greedy_decide) for many sequences at once: accepted counts and next
    tokens equal the oracle's acceptance rule at temperature 0 (go_accept: std::max_element per row, draft i+1 stands
    while row i's sample is that draft) on every sequence - with rows of tied maxima, -0.0 before +0.0, NaN first or
    inside a row, rows of NaN only; rows whose length is not a multiple of 4 and rows not on a 16-byte boundary take
    the scalar loads."""
    rng = np.random.default_rng(V + offset)
    S, k = 61, 4
    target = (rng.standard_normal((S, k + 1, V)) * 3).astype(np.float32)
    drafts = np.zeros((S, k), np.int32)
    for s_ in range(S):
        am = np.argmax(target[s_], axis=1)
        j = s_ % (k + 1)                    # the first j drafts are the rows' argmax
        drafts[s_, :j] = am[:j]
        drafts[s_, j:] = rng.integers(0, V, k - j)
    # edge rows (each on the row whose draft decides)
    target[1, 0, 7] = target[1, 0, 900] = target[1, 0].max() + 1.0           # a tie: the lower index
    drafts[1, 0] = 7
    target[2, 0, :] = 0.0
    target[2, 0, 3] = -0.0                                                 # all equal: index 0
    drafts[2, 0] = 0
    target[3, 0, 0] = np.nan                                               # NaN first: index 0
    drafts[3, 0] = 0
    target[4, 0, 5] = np.nan                                               # NaN inside: skipped
    drafts[4, 0] = int(np.nanargmax(target[4, 0]))
    target[5, 0, :] = np.nan                                               # NaN only: 0
    drafts[5, 0] = 0
    target[6, 1, :] = -np.inf                                              # -inf only: the first
    drafts[6, :2] = [int(np.argmax(target[6, 0])), 0]
    flat = np.zeros(S * (k + 1) * V + offset, np.float32)
    flat[offset:] = target.reshape(-1)
    d_flat = _dev(flat)
    d_drafts = _dev(drafts)
    scratch = torch.zeros(S * (k + 1), dtype=torch.int64, device="cuda")
    acc = torch.full((S,), -1, dtype=torch.int32, device="cuda")
    nxt = torch.full((S,), -1, dtype=torch.int32, device="cuda")
    assert L.gcuda_op_greedy_verify(_p(d_flat) + 4 * offset, _p(d_drafts), S, k, V, _p(scratch), _p(acc), _p(nxt),
                                    None) == 0
    torch.cuda.synchronize()
    acc, nxt = acc.cpu().numpy(), nxt.cpu().numpy()
    assert int(scratch.abs().sum()) == 0   # (left zeroed)
    for s_ in range(S):
        batch = np.concatenate([[0], drafts[s_]]).astype(np.int32)
        n = C.c_int(0)
        kept = O.go_accept(np.ascontiguousarray(target[s_]).ctypes.data, k + 1, V, batch.ctypes.data, 0.0, 1.0, 0,
                           C.c_uint64(0), None, 0, C.byref(n), np.zeros(k + 1, np.int32).ctypes.data)
        assert (acc[s_], nxt[s_]) == (kept - 1, n.value), s_
    assert len(set(acc.tolist())) == k + 1   # (every accepted length occurs)
    assert L.gcuda_op_greedy_verify(_p(d_flat), _p(d_drafts), 0, k, V, _p(scratch), _p(d_drafts), _p(d_drafts), None) != 0
