"""molot_attn_decode_strided_noalloc: the decode entry point for callers that
cannot allocate device memory (their runtime owns all device allocations, or
an allocation on first use would synchronise the device at a bad moment).

Its split-KV scratch is a fixed array inside the library rather than a
workspace allocated on first use.  Called through the C ABI, twice in a row
(the second call reuses the scratch the first one left behind), it must give
the same results as the allocating entry point within the parity bar.

This file is named to be collected last, so a run that stops at the first
failure has already run every other test.
"""
import ctypes

import numpy as np
import pytest

from conftest import PARITY_TOL

pytestmark = pytest.mark.gpu

_p, _i, _ll, _f = ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong, ctypes.c_float


def _noalloc(mb):
    fn = mb.library().molot_attn_decode_strided_noalloc
    fn.argtypes = [_p, _p, _p, _p, _i, _i, _i, _i, _ll, _ll, _f, _i, _i, _p]
    fn.restype = _i
    return fn


@pytest.mark.parametrize("nq,nkv,n,d,window", [
    (32, 8, 16385, 128, 0),   # 16k single-sequence decode
    (32, 8, 4097, 128, 0),
    (8, 4, 5000, 256, 1024),  # sliding window, head_dim 256
    (16, 2, 777, 64, 0),
])
def test_noalloc_matches_allocating_entry(mb, torch_cuda, orc, nq, nkv, n, d, window):
    torch = torch_cuda
    fn = _noalloc(mb)
    rng = np.random.default_rng(n + d)
    K = torch.from_numpy(rng.standard_normal((n, nkv * d)).astype(np.float32)).cuda()
    V = torch.from_numpy(rng.standard_normal((n, nkv * d)).astype(np.float32)).cuda()
    stream = torch.cuda.current_stream().cuda_stream
    scale = d ** -0.5
    for call in range(2):
        Q = torch.from_numpy(rng.standard_normal((nq, d)).astype(np.float32)).cuda()
        want = torch.empty((nq, d), device="cuda")
        mb.decode_strided(Q, K, V, want, nq, nkv, n, d, nkv * d, d, scale, n - 1, window)
        got = torch.full((nq, d), float("nan"), device="cuda")
        rc = fn(Q.data_ptr(), K.data_ptr(), V.data_ptr(), got.data_ptr(), nq, nkv, n, d, nkv * d,
                d, scale, n - 1, window, stream)
        assert rc == 0, (rc, mb.last_error())
        torch.cuda.synchronize()
        g, w = got.cpu().numpy(), want.cpu().numpy()
        assert np.all(np.isfinite(g)), call
        assert orc.rel_err(g, w) <= PARITY_TOL, call


def test_noalloc_rejects_oversize(mb, torch_cuda):
    torch = torch_cuda
    fn = _noalloc(mb)
    buf = torch.zeros(1 << 16, device="cuda")
    o = torch.zeros(1 << 12, device="cuda")
    # group 16 x head_dim 128 exceeds the fixed scratch record
    rc = fn(buf.data_ptr(), buf.data_ptr(), buf.data_ptr(), o.data_ptr(), 32, 2, 16, 128, 256,
            128, 1.0, 15, 0, None)
    assert rc == mb.ERR_UNSUPPORTED
    assert "no-alloc" in mb.last_error()
