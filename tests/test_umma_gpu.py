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
