"""The attn.h drop-ins on host buffers (synchronous, "ready on return")."""
import numpy as np
import pytest

from conftest import PARITY_TOL

pytestmark = pytest.mark.gpu


def test_attn_decode_gqa_cache_host(mb, torch_cuda, orc):
    rng = np.random.default_rng(1)
    nq, nkv, n, d = 32, 8, 4097, 128
    Q = rng.standard_normal((nq, d)).astype(np.float32)
    K = rng.standard_normal((n, nkv * d)).astype(np.float32)
    V = rng.standard_normal((n, nkv * d)).astype(np.float32)
    got = mb.attn_decode_gqa_cache(Q, K, V, nq, nkv, n, d, d ** -0.5, n - 1, 0)
    want = orc.attn_decode_gqa_cache(Q, K, V, nq, nkv, n, d, d ** -0.5, n - 1, 0)
    assert orc.rel_err(got, want) <= PARITY_TOL
    if orc.ref() is not None:
        ref = orc.attn_decode_gqa_cache(Q, K, V, nq, nkv, n, d, d ** -0.5, n - 1, 0, impl="ref")
        assert orc.rel_err(got, ref) <= PARITY_TOL


def test_attn_decode_gqa_and_win_host(mb, torch_cuda, orc):
    rng = np.random.default_rng(2)
    nq, nkv, n, d = 8, 2, 1500, 64
    Q = rng.standard_normal((nq, d)).astype(np.float32)
    K = rng.standard_normal((nkv, n, d)).astype(np.float32)
    V = rng.standard_normal((nkv, n, d)).astype(np.float32)
    got = mb.attn_decode_gqa(Q, K, V, nq, nkv, n, d, 0.125)
    want = orc.attn_decode_gqa_win(Q, K, V, nq, nkv, n, d, 0.125, n, 0)
    assert orc.rel_err(got, want) <= PARITY_TOL
    got = mb.attn_decode_gqa_win(Q, K, V, nq, nkv, n, d, 0.125, n - 1, 100)
    want = orc.attn_decode_gqa_win(Q, K, V, nq, nkv, n, d, 0.125, n - 1, 100)
    assert orc.rel_err(got, want) <= PARITY_TOL


def test_attn_decode_head_host(mb, torch_cuda, orc):
    """bench.cc:186-218 case through the drop-in, < 1e-3 of a float64 softmax."""
    import os
    z = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden",
                             "attn_head_bench.npz"))
    Q, K, V = z["Q"], z["K"], z["V"]
    n, d = K.shape
    got = mb.attn_decode_head(Q, K, V, n, d, np.float32(1.0 / np.sqrt(d)))
    assert orc.rel_err(got, z["O"]) <= PARITY_TOL
    s = (K.astype(np.float64) @ Q.astype(np.float64)) / np.sqrt(d)
    p = np.exp(s - s.max())
    assert np.max(np.abs(got - (p / p.sum()) @ V.astype(np.float64))) < 1e-3
    got = mb.attn_decode_head_win(Q, K, V, n, d, 0.1, n - 1, 40)
    want = orc.attn_decode_gqa_win(Q, K[None], V[None], 1, 1, n, d, 0.1, n - 1, 40)
    assert orc.rel_err(got, want.reshape(-1)) <= PARITY_TOL


def test_rope_apply_host(mb, torch_cuda, orc):
    rng = np.random.default_rng(3)
    for d, base, pos in ((128, 1e4, 4096), (256, 1e6, 32768), (64, 5e5, 3)):
        x = rng.standard_normal(d).astype(np.float32)
        inv = mb.rope_inv_freq(base, d)
        got = mb.rope_apply(x, d, pos, inv)
        assert orc.rel_err(got, orc.rope_apply(x, d, pos, inv)) < 1e-6


def test_zero_length_gives_zeros(mb, torch_cuda):
    Q = np.ones((4, 64), np.float32)
    K = np.zeros((0, 64), np.float32)
    got = mb.attn_decode_gqa_cache(Q, K, K, 4, 1, 0, 64, 1.0, 0, 0)
    assert not np.any(got)
