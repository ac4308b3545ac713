"""molot_attn_decode_strided_noalloc: the decode entry point for callers that
cannot allocate device memory (their runtime owns all device allocations, or
an allocation on first use would synchronise the device at a bad moment).

Its split-KV scratch is a fixed array inside the library rather than a
workspace allocated on first use.  Called through the C ABI, twice in a row
(the second call reuses the scratch the first one left behind), it must give
the same results as the allocating entry point -- bit for bit, since both
use one partition and one kernel -- and match the oracle within the parity
bar.  The cases reach the scratch limits: a partial record of group x
head_dim = 1024 and 256 kv heads (256 tickets).  A call that gives up on a
bounded wait leaves the timeout in the scratch's status word until
molot_noalloc_status reads it.

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


def _status(mb):
    fn = mb.library().molot_noalloc_status
    fn.argtypes = [_p, _i]
    fn.restype = _i
    return fn


@pytest.mark.parametrize("nq,nkv,n,d,window", [
    (32, 8, 16385, 128, 0),   # 16k single-sequence decode
    (32, 8, 4097, 128, 0),
    (8, 4, 5000, 256, 1024),  # sliding window, head_dim 256
    (16, 2, 777, 64, 0),
    (64, 8, 3000, 128, 0),    # G = 8 x head_dim 128: the largest partial record
    (16, 4, 2500, 256, 0),    # G = 4 x head_dim 256: the same record size
    (256, 256, 300, 64, 0),   # 256 kv heads: every ticket of the scratch
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
        assert np.array_equal(g, w), call
        ref = orc.attn_decode_gqa_cache(Q.cpu().numpy(), K.cpu().numpy(), V.cpu().numpy(), nq,
                                        nkv, n, d, scale, n - 1, window)
        assert orc.rel_err(g, ref) <= PARITY_TOL, call
    assert _status(mb)(stream, 1) == 0


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
    # 257 kv heads exceed the scratch's tickets
    rc = fn(buf.data_ptr(), buf.data_ptr(), buf.data_ptr(), o.data_ptr(), 257, 257, 4, 64,
            257 * 64, 64, 1.0, 3, 0, None)
    assert rc == mb.ERR_UNSUPPORTED


def test_noalloc_timeout_is_reported_then_cleared(mb, torch_cuda, orc):
    """A no-alloc call whose bounded wait runs out (molot_debug_withhold_next:
    the producer issues no copy) leaves MOLOT_ERR_TIMEOUT in the scratch's
    status word; the next call does not erase it, molot_noalloc_status
    reports it once and clears it, and calls after it are exact again."""
    torch = torch_cuda
    fn, status = _noalloc(mb), _status(mb)
    nq, nkv, n, d = 32, 8, 4097, 128
    rng = np.random.default_rng(77)
    K = torch.from_numpy(rng.standard_normal((n, nkv * d)).astype(np.float32)).cuda()
    V = torch.from_numpy(rng.standard_normal((n, nkv * d)).astype(np.float32)).cuda()
    Q = torch.from_numpy(rng.standard_normal((nq, d)).astype(np.float32)).cuda()
    stream = torch.cuda.current_stream().cuda_stream
    out = torch.empty((nq, d), device="cuda")
    args = (Q.data_ptr(), K.data_ptr(), V.data_ptr(), out.data_ptr(), nq, nkv, n, d, nkv * d, d,
            d ** -0.5, n - 1, 0, stream)
    assert status(stream, 1) == 0
    mb.debug_withhold_next(2_000_000)
    assert fn(*args) == 0
    assert fn(*args) == 0  # a normal call after it leaves the word alone
    assert status(stream, 0) == mb.ERR_TIMEOUT
    assert mb.device_status(clear=False) == mb.ERR_TIMEOUT
    assert status(stream, 1) == mb.ERR_TIMEOUT
    assert status(stream, 1) == 0
    for _ in range(2):
        out.fill_(float("nan"))
        assert fn(*args) == 0
        assert status(stream, 1) == 0
        want = orc.attn_decode_gqa_cache(Q.cpu().numpy(), K.cpu().numpy(), V.cpu().numpy(), nq,
                                         nkv, n, d, d ** -0.5, n - 1, 0)
        assert orc.rel_err(out.cpu().numpy(), want) <= PARITY_TOL
