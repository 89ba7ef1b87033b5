"""The tensor-core (tcgen05) q4 product (gcuda_op_q4_gemm_umma on the U layout of gcuda_op_q4_umma_relayout) against
the oracle's matvec_rows_q_ref (engine/src/kernels.cpp:1304-1322), itself pinned to the reference: every output bit
for bit, at the verify step's shapes (1..8 token rows, the expert and projection matrices) and at many token rows
(several token blocks of the kernel, as the batched configuration's grouped expert products take). The kernel's
bounded waits must not have given up (the operators' status word stays 0)."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from geode_b200 import cuda_lib, synth  # noqa: E402
import oracle_py as op  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def L():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    return cuda_lib()


@pytest.fixture(scope="module")
def O():
    return op.oracle_lib()


def _u(L, packed, rows, cols):
    d_pack = torch.from_numpy(np.ascontiguousarray(packed)).cuda()
    nb = L.gcuda_op_q4_umma_bytes(rows, cols)
    assert nb == rows * cols // 16 * 9
    d_u = torch.zeros(nb, dtype=torch.uint8, device="cuda")
    assert L.gcuda_op_q4_umma_relayout(d_pack.data_ptr(), rows, cols, d_u.data_ptr(), None) == 0
    return d_u


@pytest.mark.parametrize("rows,cols,n", [(128, 256, 1), (1024, 2048, 5), (2048, 512, 3), (256, 2048, 8),
                                         (512, 2048, 4), (384, 1024, 40), (128, 2048, 100)])
def test_umma_gemm_bit_exact(L, O, rows, cols, n):
    rng = np.random.default_rng(rows * 7 + cols + n)
    packed, g = synth.q4_random(rng, rows, cols)
    d_u = _u(L, packed, rows, cols)
    x = (rng.standard_normal((n, cols)) * rng.uniform(0.5, 3.0, (n, 1))).astype(np.float32)
    x[0, :16] = 0.0   # an all-zero activation block
    d_x = torch.from_numpy(x).cuda()
    q = torch.zeros((n, cols), dtype=torch.int8, device="cuda")
    s = torch.zeros((n, cols // 16), dtype=torch.float32, device="cuda")
    b = torch.zeros((n, cols // 16), dtype=torch.int32, device="cuda")
    assert L.gcuda_op_quantize(d_x.data_ptr(), n, cols, q.data_ptr(), s.data_ptr(), b.data_ptr(), None) == 0
    y = torch.full((n, rows), float("nan"), dtype=torch.float32, device="cuda")
    assert L.gcuda_op_q4_gemm_umma(d_u.data_ptr(), rows, cols, g, q.data_ptr(), s.data_ptr(), b.data_ptr(), n,
                                   y.data_ptr(), None) == 0
    torch.cuda.synchronize()
    assert L.gcuda_op_status(1) == 0
    ref = op.oracle_matvec_q(O, packed, rows, cols, g, x)
    got = y.cpu().numpy()
    bad = np.argwhere(got.view(np.uint32) != ref.view(np.uint32))
    assert bad.size == 0, (len(bad), bad[:5], got[tuple(bad[0])], ref[tuple(bad[0])])


def test_umma_shapes_refused(L):
    assert L.gcuda_op_q4_umma_bytes(100, 256) == 0 and L.gcuda_op_q4_umma_bytes(128, 320) == 0
    d = torch.zeros(1024, dtype=torch.uint8, device="cuda")
    assert L.gcuda_op_q4_gemm_umma(d.data_ptr(), 100, 256, 1.0, d.data_ptr(), d.data_ptr(), d.data_ptr(), 1,
                                   d.data_ptr(), None) != 0


@pytest.mark.parametrize("n,K,E,H,ff", [(20, 4, 16, 512, 256), (64, 8, 64, 2048, 512)])
def test_moe_umma_bit_exact(L, O, n, K, E, H, ff):
    """The routed experts of many rows on the tensor core (gcuda_op_moe_umma: the picks grouped by expert on the device,
    the grouped gate_up, SwiGLU + quantize, the grouped down) against the oracle's per-pick expert products
    (go_expert_pair, the reference's Model::moe pick, engine/src/model.cpp:4496-4543): every output row bit for bit.
    The picks lean on a few experts (Zipf-like), so units of several token blocks and single picks both occur."""
    import ctypes as C
    rng = np.random.default_rng(n + E)
    gu_rows = 2 * ff
    blocks, globs = [], []
    for e in range(E):
        gu, g0 = synth.q4_random(rng, gu_rows, H)
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
    eb = L.gcuda_op_moe_umma_expert_bytes(H, ff)
    assert eb == stride
    d_pack = torch.from_numpy(pack).cuda()
    d_u = torch.zeros(E * eb, dtype=torch.uint8, device="cuda")
    assert L.gcuda_op_moe_umma_relayout(d_pack.data_ptr(), stride, E, H, ff, d_u.data_ptr(), None) == 0
    d_h = torch.from_numpy(h).cuda()
    q = torch.zeros((n, H), dtype=torch.int8, device="cuda")
    s = torch.zeros((n, H // 16), dtype=torch.float32, device="cuda")
    b = torch.zeros((n, H // 16), dtype=torch.int32, device="cuda")
    assert L.gcuda_op_quantize(d_h.data_ptr(), n, H, q.data_ptr(), s.data_ptr(), b.data_ptr(), None) == 0
    wb = L.gcuda_op_moe_umma_work_bytes(n, K, E, H, ff)
    work = torch.zeros(wb, dtype=torch.uint8, device="cuda")
    out = torch.full((n * K, H), float("nan"), dtype=torch.float32, device="cuda")
    d_ids = torch.from_numpy(ids).cuda()
    d_g = torch.from_numpy(globs).cuda()
    for rep in range(2):   # (twice: the work buffer's plan from the first call is overwritten cleanly)
        assert L.gcuda_op_moe_umma(d_u.data_ptr(), d_g.data_ptr(), E, H, ff, q.data_ptr(), s.data_ptr(), b.data_ptr(), n,
                                   d_ids.data_ptr(), K, out.data_ptr(), work.data_ptr(), wb, None) == 0
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
