"""GPU parity of the Q4 GEMV (gemm.h:223-254, the projections around the
attention path) against the reference's golden vectors and the oracle."""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
# Same integer group sums; the float sum over groups is reassociated (lanes,
# then a warp tree) where the reference adds them in order.
GEMV_TOL = 1e-6


def test_gemv_q4_against_reference_golden(mb, torch_cuda, orc):
    z = np.load(os.path.join(GOLDEN, "gemv_q4.npz"))
    for name in ("gemv_a", "gemv_b"):
        q4 = tuple(z[f"{name}/{k}"] for k in ("scales", "zeros", "data", "wsums"))
        y = mb.gemv_q4(q4, z[f"{name}/x"])
        assert orc.rel_err(y, z[f"{name}/y"]) < GEMV_TOL, name


@pytest.mark.parametrize("rows,cols", [(4096, 4096), (1024, 4096), (14336, 4096), (4096, 14336),
                                       (3, 32), (100, 96), (257, 1056)])
def test_gemv_q4_dev_against_oracle(mb, torch_cuda, orc, rows, cols):
    torch = torch_cuda
    rng = np.random.default_rng(rows + cols)
    W = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
    W[0, :32] = 0.0  # a flat group
    q4 = orc.quantize_q4(W)
    x = (rng.standard_normal(cols) * rng.uniform(0.1, 10)).astype(np.float32)
    x[32:64] = 0.0  # an all-zero activation block
    want = orc.gemv_q4(q4, x)
    dev = [torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in q4[:3]]
    y = torch.full((rows,), float("nan"), device="cuda")
    mb.gemv_q4_dev(dev[0], dev[1], dev[2], torch.from_numpy(x).cuda(), y)
    torch.cuda.synchronize()
    assert orc.rel_err(y.cpu().numpy(), want) < GEMV_TOL


def test_gemv_q4_rejects_bad_shapes(mb, torch_cuda):
    sc = np.zeros((2, 1), np.float32)
    z = np.zeros((2, 1), np.int8)
    d = np.zeros((2, 16), np.uint8)
    with pytest.raises(mb.MolotError):
        mb._lib and mb.check(mb._lib.molot_gemv_q4(mb._ptr(sc), mb._ptr(z), mb._ptr(d), None, 2, 33,
                                                   mb._ptr(np.zeros(33, np.float32)),
                                                   mb._ptr(np.zeros(2, np.float32))))
