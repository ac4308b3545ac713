"""GPU parity of the split-KV decode kernel against the CPU oracle.

Bar: max|gpu - ref| / max|ref| <= 1e-5 per output,
where ref is the restatement of attn.h:125-177 that is bit-exact with the
reference.  Each case also checks that the GPU's error against a float64
evaluation is no larger than the reference's own (plus 1e-6).
"""
import numpy as np
import pytest

from conftest import PARITY_TOL

pytestmark = pytest.mark.gpu


def _inputs(nq, nkv, n, d, seed):
    rng = np.random.default_rng(seed)
    Q = rng.standard_normal((nq, d)).astype(np.float32)
    K = rng.standard_normal((n, nkv * d)).astype(np.float32)
    V = rng.standard_normal((n, nkv * d)).astype(np.float32)
    return Q, K, V


def _gpu_cache(mb, torch, Q, K, V, nq, nkv, n, d, scale, pos, window):
    dq = torch.from_numpy(Q).cuda()
    dk = torch.from_numpy(K).cuda()
    dv = torch.from_numpy(V).cuda()
    do = torch.full((nq, d), float("nan"), device="cuda")
    mb.decode_strided(dq, dk, dv, do, nq, nkv, n, d, nkv * d, d, scale, pos, window)
    torch.cuda.synchronize()
    assert mb.device_status() == 0
    return do.cpu().numpy()


def _check(orc, got, Q, K, V, nq, nkv, n, d, scale, pos, window):
    want = orc.attn_decode_gqa_cache(Q, K, V, nq, nkv, n, d, scale, pos, window)
    f64 = orc.attn_decode_gqa_cache_f64(Q, K, V, nq, nkv, n, d, scale, pos, window)
    assert np.all(np.isfinite(got))
    e_ref = orc.rel_err(got, want)
    e_gpu64 = orc.rel_err(got, f64)
    e_ref64 = orc.rel_err(want, f64)
    assert e_ref <= PARITY_TOL, (e_ref, e_gpu64, e_ref64)
    assert e_gpu64 <= 1.1 * e_ref64 + 1e-6, (e_ref, e_gpu64, e_ref64)
    return e_ref


# (nq, nkv, n, d, scale, window): the BASELINE configs at full size, then edges.
FULL = [
    (32, 8, 4097, 128, 128 ** -0.5, 0),          # cfg1
    (32, 8, 16385, 128, 128 ** -0.5, 0),         # cfg2
    (8, 4, 32769, 256, 1.0 / 16, 0),             # cfg3 global layer, scale 1/sqrt(d)
    (8, 4, 32769, 256, 1.0, 0),                  # cfg3 global layer, attn_scale_one
    (8, 4, 32769, 256, 1.0, 1024),               # cfg3 sliding-window layer
    (64, 8, 8192, 128, 128 ** -0.5, 0),          # cfg5 head shape
]


@pytest.mark.parametrize("case", FULL, ids=lambda c: f"nq{c[0]}_nkv{c[1]}_n{c[2]}_d{c[3]}_w{c[5]}")
def test_baseline_configs(mb, torch_cuda, orc, case):
    nq, nkv, n, d, scale, window = case
    Q, K, V = _inputs(nq, nkv, n, d, seed=n + d)
    got = _gpu_cache(mb, torch_cuda, Q, K, V, nq, nkv, n, d, scale, n - 1, window)
    _check(orc, got, Q, K, V, nq, nkv, n, d, scale, n - 1, window)


@pytest.mark.parametrize("n", [1, 2, 7, 15, 16, 17, 31, 63, 64, 65, 127, 128, 129, 255, 1000])
def test_edge_lengths(mb, torch_cuda, orc, n):
    nq, nkv, d = 32, 8, 128
    Q, K, V = _inputs(nq, nkv, n, d, seed=n)
    got = _gpu_cache(mb, torch_cuda, Q, K, V, nq, nkv, n, d, 0.088, n - 1, 0)
    _check(orc, got, Q, K, V, nq, nkv, n, d, 0.088, n - 1, 0)


@pytest.mark.parametrize("d,group", [(64, 1), (64, 2), (64, 4), (64, 8), (64, 16), (64, 32),
                                     (128, 1), (128, 2), (128, 4), (128, 8), (128, 16),
                                     (128, 32), (256, 1), (256, 2), (256, 4), (256, 8),
                                     (256, 16)])
def test_head_dims_and_groups(mb, torch_cuda, orc, d, group):
    nkv = 2
    nq = nkv * group
    n = 777
    Q, K, V = _inputs(nq, nkv, n, d, seed=d * 100 + group)
    scale = d ** -0.5
    got = _gpu_cache(mb, torch_cuda, Q, K, V, nq, nkv, n, d, scale, n - 1, 0)
    _check(orc, got, Q, K, V, nq, nkv, n, d, scale, n - 1, 0)


@pytest.mark.parametrize("n,pos,window", [
    (300, 299, 1),      # only the newest slot
    (300, 299, 16),     # window ends a block boundary away
    (300, 299, 17),
    (300, 299, 300),    # window == n: everything
    (300, 299, 5000),   # window > n
    (300, 150, 40),     # pos inside the cache: slots [111, 300) (t0 from pos, end at n)
    (4096, 4095, 1024), # cfg3-style SWA
    (50, 80, 20),       # t0 = 61 >= n: empty range -> zeros
])
def test_windows(mb, torch_cuda, orc, n, pos, window):
    nq, nkv, d = 8, 2, 128
    Q, K, V = _inputs(nq, nkv, n, d, seed=pos + window)
    got = _gpu_cache(mb, torch_cuda, Q, K, V, nq, nkv, n, d, 0.1, pos, window)
    t0 = pos - window + 1 if window > 0 and pos - window + 1 > 0 else 0
    if t0 >= n:
        assert not np.any(got)
        want = orc.attn_decode_gqa_cache(Q, K, V, nq, nkv, n, d, 0.1, pos, window)
        assert not np.any(want)
    else:
        _check(orc, got, Q, K, V, nq, nkv, n, d, 0.1, pos, window)


def test_single_slot_returns_value_row(mb, torch_cuda):
    nq, nkv, d = 8, 2, 128
    Q, K, V = _inputs(nq, nkv, 1, d, seed=3)
    got = _gpu_cache(mb, torch_cuda, Q, K, V, nq, nkv, 1, d, 0.1, 0, 0)
    want = np.repeat(V.reshape(nkv, d), nq // nkv, axis=0)
    assert np.array_equal(got, want)


def test_head_major_layout(mb, torch_cuda, orc):
    """attn.h:111 layout [nkv][n][d] through the strided entry point."""
    torch = torch_cuda
    nq, nkv, n, d = 16, 4, 3000, 128
    rng = np.random.default_rng(9)
    Q = rng.standard_normal((nq, d)).astype(np.float32)
    Kh = rng.standard_normal((nkv, n, d)).astype(np.float32)
    Vh = rng.standard_normal((nkv, n, d)).astype(np.float32)
    do = torch.empty((nq, d), device="cuda")
    mb.decode_strided(torch.from_numpy(Q).cuda(), torch.from_numpy(Kh).cuda(),
                      torch.from_numpy(Vh).cuda(), do, nq, nkv, n, d, d, n * d, 0.09, n - 1, 0)
    torch.cuda.synchronize()
    want = orc.attn_decode_gqa_win(Q, Kh, Vh, nq, nkv, n, d, 0.09, n - 1, 0)
    assert orc.rel_err(do.cpu().numpy(), want) <= PARITY_TOL


def test_repeat_calls_bitwise_stable(mb, torch_cuda):
    """Tickets reset between launches and the combine order is fixed."""
    torch = torch_cuda
    nq, nkv, n, d = 32, 8, 20000, 128
    Q, K, V = _inputs(nq, nkv, n, d, seed=5)
    a = _gpu_cache(mb, torch, Q, K, V, nq, nkv, n, d, 0.088, n - 1, 0)
    b = _gpu_cache(mb, torch, Q, K, V, nq, nkv, n, d, 0.088, n - 1, 0)
    assert np.array_equal(a.view(np.int32), b.view(np.int32))


def test_unaligned_cache_rejected(mb, torch_cuda):
    torch = torch_cuda
    nq, nkv, n, d = 8, 2, 64, 128
    buf = torch.zeros(n * nkv * d + 1, device="cuda")
    q = torch.zeros(nq * d, device="cuda")
    o = torch.zeros(nq * d, device="cuda")
    with pytest.raises(mb.MolotError) as ei:
        mb.decode_strided(q, buf[1:], buf[1:], o, nq, nkv, n, d, nkv * d, d, 0.1, n - 1, 0)
    assert ei.value.status == mb.ERR_INVALID
