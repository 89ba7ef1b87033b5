"""The verify step's expert kernels (k_experts_lane: a lane a weight row, dp4a on the codes for only the tokens that
picked each expert, the reference's block chain in that lane) through their operators (gcuda_op_moe_lane_relayout,
gcuda_op_moe_lane) against the oracle's per-pick expert products (go_expert_pair, the reference's Model::moe pick,
engine/src/model.cpp:4496-4543, pinned to the reference): every output row bit for bit - the gate_up product, the
SwiGLU and its quantization, the down product. At the benchmark's own expert shape (256 experts, hidden 2048, expert
ff 512, 5 rows x top-8), a smaller one, and a narrow one whose K takes the kernels' one-group stages. The picks lean on a
few experts (Zipf-like), so members with several tokens occur beside single picks. The kernels' bounded waits must
not have given up (the operators' status word stays 0)."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from geode_b200 import synth  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def L():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    from geode_b200 import cuda_lib
    return cuda_lib()


@pytest.fixture(scope="module")
def O():
    import oracle_py as op
    return op.oracle_lib()


@pytest.mark.parametrize("n,K,E,H,ff", [(5, 8, 256, 2048, 512), (5, 8, 64, 1024, 256), (3, 4, 16, 256, 128)])
def test_moe_lane_bit_exact(L, O, n, K, E, H, ff):
    rng = np.random.default_rng(n * 7 + E)
    blocks, globs = [], []
    for e in range(E):
        gu, g0 = synth.q4_random(rng, 2 * ff, H)
        dn, g1 = synth.q4_random(rng, H, ff)
        blocks.append(np.concatenate([gu.reshape(-1), dn.reshape(-1)]))
        globs.append((g0, g1))
    pack = np.ascontiguousarray(np.stack(blocks))
    stride = pack.shape[1]
    globs = np.array(globs, np.float32)
    p_e = 1.0 / np.arange(1, E + 1)
    p_e /= p_e.sum()
    ids = np.stack([rng.choice(E, K, replace=False, p=p_e) for _ in range(n)]).astype(np.int32)
    h = (rng.standard_normal((n, H)) * rng.uniform(0.5, 2.0, (n, 1))).astype(np.float32)
    eb = L.gcuda_op_moe_lane_expert_bytes(H, ff)
    assert eb == stride
    d_pack = torch.from_numpy(pack).cuda()
    d_r16 = torch.zeros(E * eb, dtype=torch.uint8, device="cuda")
    assert L.gcuda_op_moe_lane_relayout(d_pack.data_ptr(), stride, E, H, ff, d_r16.data_ptr(), None) == 0
    d_h = torch.from_numpy(h).cuda()
    q = torch.zeros((n, H), dtype=torch.int8, device="cuda")
    s = torch.zeros((n, H // 16), dtype=torch.float32, device="cuda")
    b = torch.zeros((n, H // 16), dtype=torch.int32, device="cuda")
    assert L.gcuda_op_quantize(d_h.data_ptr(), n, H, q.data_ptr(), s.data_ptr(), b.data_ptr(), None) == 0
    wb = L.gcuda_op_moe_lane_work_bytes(n, K, H, ff)
    assert wb > 0
    work = torch.zeros(wb, dtype=torch.uint8, device="cuda")
    out = torch.full((n * K, H), float("nan"), dtype=torch.float32, device="cuda")
    d_ids = torch.from_numpy(ids).cuda()
    d_g = torch.from_numpy(globs).cuda()
    for rep in range(2):   # (twice: the work buffer's route from the first call is overwritten cleanly)
        assert L.gcuda_op_moe_lane(d_r16.data_ptr(), d_g.data_ptr(), E, H, ff, q.data_ptr(), s.data_ptr(), b.data_ptr(),
                                   n, d_ids.data_ptr(), K, out.data_ptr(), work.data_ptr(), wb, None) == 0
        torch.cuda.synchronize()
        assert L.gcuda_op_status(1) == 0
    got = out.cpu().numpy()
    for t in range(n):
        for k in range(K):
            e = int(ids[t, k])
            ref = np.zeros(H, np.float32)
            O.go_expert_pair(pack[e].ctypes.data, float(globs[e, 0]), float(globs[e, 1]), H, ff, h[t].ctypes.data,
                             ref.ctypes.data)
            row = got[t * K + k]
            assert np.array_equal(row.view(np.uint32), ref.view(np.uint32)), (t, k, e, np.abs(row - ref).max())


def test_moe_lane_refusals(L):
    """Shapes the kernels do not take are refused before anything runs: more than 8 rows or picks, widths off 64."""
    assert L.gcuda_op_moe_lane_work_bytes(9, 8, 2048, 512) == 0
    assert L.gcuda_op_moe_lane_work_bytes(5, 9, 2048, 512) == 0
    assert L.gcuda_op_moe_lane_work_bytes(5, 8, 2000, 512) == 0
    assert L.gcuda_op_moe_lane_expert_bytes(2048, 500) == 0
