"""GPU parity of causal / sliding-window prefill attention (gemm.h:409-446,
forward.h:368-398) against the reference's golden vectors and the oracle."""
import math
import os

import numpy as np
import pytest

from conftest import PARITY_TOL

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def cu(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def test_prefill_host_dropin_against_reference_golden(mb, torch_cuda, orc):
    z = np.load(os.path.join(GOLDEN, "prefill.npz"))
    for name in sorted({k.split("/")[0] for k in z.files}):
        nq, nkv, d, M, N, pos0, window = (int(x) for x in z[f"{name}/params"])
        got = mb.attn_prefill_gqa(z[f"{name}/Q"], z[f"{name}/K"], z[f"{name}/V"], nq, nkv, M, N,
                                  d, float(z[f"{name}/scale"]), pos0, window)
        assert orc.rel_err(got, z[f"{name}/O"]) <= PARITY_TOL, name


@pytest.mark.parametrize("nq,nkv,d,M,pos0,N_extra,window", [
    (32, 8, 128, 300, 0, 0, 0),       # cfg1 shape, prompt from an empty cache
    (32, 8, 128, 77, 500, 0, 0),      # continuation after 500 cached slots
    (8, 4, 256, 150, 900, 0, 1024),   # gemma SWA layer
    (8, 4, 256, 90, 1200, 0, 64),     # window shorter than the prompt
    (16, 16, 64, 70, 3, 0, 0),        # G = 1
    (32, 2, 64, 45, 10, 0, 5),        # G = 16, tiny window
    (64, 8, 128, 33, 20, 0, 0),       # G = 8 (Llama-70B shape)
    (8, 2, 128, 40, 30, -25, 0),      # cache shorter than the positions (nn = N)
    (8, 2, 128, 1, 63, 0, 0),         # one token
    (32, 8, 128, 600, 200, 0, 256),   # many key tiles, window spanning tiles (tensor-core path)
    (16, 4, 64, 257, 1000, -200, 0),  # head_dim 64, ragged last query block, nn = N
])
def test_prefill_strided_against_oracle(mb, torch_cuda, orc, nq, nkv, d, M, pos0, N_extra,
                                        window):
    torch = torch_cuda
    rng = np.random.default_rng(M * 7 + pos0)
    N = pos0 + M + N_extra
    Q = rng.standard_normal((M, nq, d)).astype(np.float32)
    K = rng.standard_normal((N, nkv * d)).astype(np.float32)
    V = rng.standard_normal((N, nkv * d)).astype(np.float32)
    scale = d ** -0.5
    want = orc.attn_prefill_gqa(Q, K, V, nq, nkv, M, N, d, scale, pos0, window)
    O = torch.full((M, nq, d), float("nan"), device="cuda")
    # slot-major [N][nkv*d] as attn.h stores it
    mb.prefill_strided(cu(torch, Q), cu(torch, K), cu(torch, V), O, nq, nkv, M, N, d, nkv * d, d,
                       scale, pos0, window)
    torch.cuda.synchronize()
    assert orc.rel_err(O.cpu().numpy(), want) <= PARITY_TOL
    # head-major [nkv][N][d], the KV handle's layout
    Kh = np.ascontiguousarray(K.reshape(N, nkv, d).transpose(1, 0, 2))
    Vh = np.ascontiguousarray(V.reshape(N, nkv, d).transpose(1, 0, 2))
    O2 = torch.full((M, nq, d), float("nan"), device="cuda")
    mb.prefill_strided(cu(torch, Q), cu(torch, Kh), cu(torch, Vh), O2, nq, nkv, M, N, d, d,
                       N * d, scale, pos0, window)
    torch.cuda.synchronize()
    assert np.array_equal(O.cpu().numpy(), O2.cpu().numpy())


def test_prefill_through_the_handle_then_decode(mb, torch_cuda, orc):
    """forward.h:368-398 then forward.h:554-590: a prompt of M tokens is
    normalised, rotated, appended and attended in two launches; the next
    token is a fused decode step over the prefilled cache."""
    torch = torch_cuda
    nq, nkv, hd, M, cap = 8, 4, 256, 100, 128
    rng = np.random.default_rng(3)
    q = rng.standard_normal((M, nq, hd)).astype(np.float32)
    k = rng.standard_normal((M, nkv, hd)).astype(np.float32)
    v = rng.standard_normal((M, nkv, hd)).astype(np.float32)
    qn = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    kn = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    freq = orc.rope_inv_freq(1e4, hd)
    window = 48
    kv = mb.KVCache(1, nkv, hd, cap)
    try:
        q_rot = torch.empty((M, nq, hd), device="cuda")
        out = torch.empty((M, nq, hd), device="cuda")
        kv.append_rope_tokens(0, cu(torch, q), cu(torch, k), cu(torch, v), q_rot, cu(torch, qn),
                              cu(torch, kn), True, 1e-6, cu(torch, freq), 0)
        kv.prefill(0, q_rot, out, 1.0, 0, window)
        kv.check()
        assert kv.length(0) == M
        # the oracle replays forward.h's per-token prologue then the prefill
        qr = np.empty_like(q)
        kc = np.zeros((cap, nkv * hd), np.float32)
        vc = np.zeros_like(kc)
        for m in range(M):
            for h in range(nq):
                qr[m, h] = orc.rope_apply(orc.rmsnorm(q[m, h], qn, 1e-6), hd, m, freq)
            for h in range(nkv):
                kc[m, h * hd:(h + 1) * hd] = orc.rope_apply(orc.rmsnorm(k[m, h], kn, 1e-6), hd, m,
                                                            freq)
            vc[m] = orc.rmsnorm_plain(v[m].reshape(-1), 1e-6)
        assert orc.rel_err(q_rot.cpu().numpy(), qr) < 1e-6
        kt, vt = kv.layer_tensors(0)
        assert orc.rel_err(kt[:, :M].permute(1, 0, 2).reshape(M, -1).cpu().numpy(), kc[:M]) < 1e-6
        assert orc.rel_err(vt[:, :M].permute(1, 0, 2).reshape(M, -1).cpu().numpy(), vc[:M]) < 1e-6
        want = orc.attn_prefill_gqa(qr, kc, vc, nq, nkv, M, M, hd, 1.0, 0, window)
        assert orc.rel_err(out.cpu().numpy(), want) <= PARITY_TOL
        # query m of the prefill == a decode at position m over slots [0, m]
        for m in (0, 17, M - 1):
            dec = orc.attn_decode_gqa_cache(qr[m].reshape(-1), kc, vc, nq, nkv, m + 1, hd, 1.0, m,
                                            window)
            assert orc.rel_err(out[m].cpu().numpy(), dec) <= PARITY_TOL, m
        # next token: one fused step over the prefilled cache
        q1 = rng.standard_normal(nq * hd).astype(np.float32)
        k1 = rng.standard_normal(nkv * hd).astype(np.float32)
        v1 = rng.standard_normal(nkv * hd).astype(np.float32)
        o1 = torch.empty(nq * hd, device="cuda")
        kv.step(0, cu(torch, q1), cu(torch, k1), cu(torch, v1), o1, 1.0, M, window,
                cu(torch, qn), cu(torch, kn), True, 1e-6, cu(torch, freq))
        kv.check()
        st, n1, want1 = orc.attn_layer_step(q1.copy(), k1.copy(), v1.copy(), qn, kn, 1, 1e-6,
                                            freq, M, kc, vc, M, (nq, hd), nq, nkv, hd, 1.0,
                                            window)
        assert st == 0 and n1 == M + 1
        assert orc.rel_err(o1.cpu().numpy().reshape(nq, hd), want1) <= PARITY_TOL
    finally:
        kv.close()


def test_prefill_errors(mb, torch_cuda):
    torch = torch_cuda
    kv = mb.KVCache(1, 2, 64, 10)
    try:
        x = torch.zeros((8, 6, 64), device="cuda")
        kk = torch.zeros((8, 2, 64), device="cuda")
        with pytest.raises(mb.MolotError) as ei:  # 8 tokens fit, 11 do not
            kv.append_rope_tokens(0, torch.zeros((11, 6, 64), device="cuda"),
                                  torch.zeros((11, 2, 64), device="cuda"),
                                  torch.zeros((11, 2, 64), device="cuda"),
                                  torch.zeros((11, 6, 64), device="cuda"))
        assert ei.value.status == mb.ERR_CACHE_FULL
        kv.append_rope_tokens(0, x, kk, kk, x.clone())
        with pytest.raises(mb.MolotError) as ei:  # group 3 does not divide 64
            kv.prefill(0, x, x.clone(), 1.0, 0)
        assert ei.value.status == mb.ERR_UNSUPPORTED
        kv.check()
    finally:
        kv.close()
    Q = np.zeros((4, 4, 64), np.float32)
    K = np.zeros((4, 2 * 64), np.float32)
    empty = mb.attn_prefill_gqa(Q, K, K, 4, 2, 4, 0, 64, 1.0, 0, 0)  # N = 0: zeros
    assert not np.any(empty) and not math.isnan(float(empty.sum()))
