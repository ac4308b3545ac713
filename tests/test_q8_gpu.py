"""Q8 KV-cache storage (MOLOT_KV_Q8): every row entering the cache is stored
as int8 codes with one FP32 scale per 32 values (the reference's Q8 block
rule, quant.h:33-43); the attention math stays FP32 on the values read back
as code * scale.  The parity contract: the cache bytes equal the oracle's
quantization of the same rows bit for bit, and the attention output matches
the reference's algorithm run on the dequantized cache within the 1e-5 bar
(the kernel reads a lane's four dims of each 32-value block from one word,
which reorders the score sums at rounding level)."""
import numpy as np
import pytest

from conftest import PARITY_TOL

pytestmark = pytest.mark.gpu


def cu(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def cache_rows(mb, t, n, hd):
    """[nkv][cap][row] uint8 cache view -> (codes [n][nkv][hd], scales [n][nkv][hd/32])."""
    raw = t[:, :n].permute(1, 0, 2).contiguous().cpu().numpy()
    return mb.q8_unpack(raw, hd)


def oracle_q8(orc, rows, nkv, hd):
    """[n][nkv*hd] float32 rows -> (codes, scales, dequantized [n][nkv*hd])."""
    q, s = orc.quantize_q8_blocks(np.asarray(rows, np.float32).reshape(-1, nkv, hd))
    return q, s, orc.dequantize_q8_blocks(q, s).reshape(len(rows), nkv * hd)


def assert_cache_equals(mb, orc, kv, layer, n, K, V):
    kt, vt = kv.layer_tensors(layer)
    for t, rows in ((kt, K), (vt, V)):
        q, s = cache_rows(mb, t, n, kv.hd)
        wq, ws, _ = oracle_q8(orc, rows, kv.nkv, kv.hd)
        assert np.array_equal(q, wq)
        assert np.array_equal(s.view(np.uint32), ws.view(np.uint32))


def test_row_layout(mb, torch_cuda):
    assert mb.q8_row_bytes(128) == 144 and mb.q8_row_bytes(256) == 288
    assert mb.q8_row_bytes(64) == 80
    kv = mb.KVCache(1, 2, 128, 8, dtype="q8")
    try:
        kt, _ = kv.layer_tensors(0)
        assert tuple(kt.shape) == (2, 8, 144) and str(kt.dtype) == "torch.uint8"
    finally:
        kv.close()


def test_write_quantizes_rows(mb, torch_cuda, orc):
    torch = torch_cuda
    rng = np.random.default_rng(2)
    nkv, hd, cap, n = 4, 128, 40, 33
    k = (rng.standard_normal((n, nkv * hd)) * rng.uniform(0.01, 50, (n, 1))).astype(np.float32)
    v = rng.standard_normal((n, nkv * hd)).astype(np.float32)
    k[4, :32] = 0.0  # an all-zero block: scale 1, codes 0
    kv = mb.KVCache(2, nkv, hd, cap, dtype="q8")
    try:
        kv.write(0, 3, k, v)                       # host rows
        kv.write(1, 0, cu(torch, k), cu(torch, v))  # device rows
        kv.check()
        for layer, s0 in ((0, 3), (1, 0)):
            kt, vt = kv.layer_tensors(layer)
            for t, rows in ((kt, k), (vt, v)):
                raw = t[:, s0:s0 + n].permute(1, 0, 2).contiguous().cpu().numpy()
                q, s = mb.q8_unpack(raw, hd)
                wq, ws, _ = oracle_q8(orc, rows, nkv, hd)
                assert np.array_equal(q, wq) and np.array_equal(s, ws)
    finally:
        kv.close()


@pytest.mark.parametrize("nq,nkv,hd,n,window", [
    (32, 8, 128, 4097, 0),    # cfg1 shape
    (32, 8, 128, 16385, 0),   # cfg2 shape
    (8, 4, 256, 3000, 1024),  # gemma SWA layer
    (64, 8, 64, 777, 0),      # G = 8, d = 64
    (4, 4, 128, 17, 0),       # G = 1, ragged
    (64, 2, 128, 300, 0),     # G = 32
    (32, 2, 256, 200, 64),    # G = 16, d = 256, window
])
def test_decode_on_q8_cache(mb, torch_cuda, orc, nq, nkv, hd, n, window):
    torch = torch_cuda
    rng = np.random.default_rng(n + hd + nq)
    k = rng.standard_normal((n, nkv * hd)).astype(np.float32)
    v = rng.standard_normal((n, nkv * hd)).astype(np.float32)
    q = rng.standard_normal(nq * hd).astype(np.float32)
    kv = mb.KVCache(1, nkv, hd, n, dtype="q8")
    try:
        kv.write(0, 0, cu(torch, k), cu(torch, v))
        kv.set_length(0, n)
        o = torch.full((nq * hd,), float("nan"), device="cuda")
        kv.decode(0, cu(torch, q), o, hd ** -0.5, n - 1, window)
        kv.check()
        _, _, kd = oracle_q8(orc, k, nkv, hd)
        _, _, vd = oracle_q8(orc, v, nkv, hd)
        want = orc.attn_decode_gqa_cache(q, kd, vd, nq, nkv, n, hd, hd ** -0.5, n - 1, window)
        assert orc.rel_err(o.cpu().numpy().reshape(nq, hd), want) <= PARITY_TOL
    finally:
        kv.close()


@pytest.mark.parametrize("nq,nkv,hd,n0,window", [(32, 8, 128, 5000, 0), (8, 4, 256, 900, 256),
                                                 (16, 2, 64, 63, 0)])
def test_fused_step_on_q8_cache(mb, torch_cuda, orc, nq, nkv, hd, n0, window):
    """One launch (step) == append + decode bit for bit; the new row's codes
    equal the oracle's quantization of the reference prologue's row."""
    torch = torch_cuda
    rng = np.random.default_rng(n0 + 1)
    cap = n0 + 2
    kc = rng.standard_normal((n0, nkv * hd)).astype(np.float32)
    vc = rng.standard_normal((n0, nkv * hd)).astype(np.float32)
    q = rng.standard_normal(nq * hd).astype(np.float32)
    k = rng.standard_normal(nkv * hd).astype(np.float32)
    v = rng.standard_normal(nkv * hd).astype(np.float32)
    qn = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    kn = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    freq = orc.rope_inv_freq(1e4, hd)
    outs = []
    for fused in (True, False):
        kv = mb.KVCache(1, nkv, hd, cap, dtype="q8")
        try:
            kv.write(0, 0, cu(torch, kc), cu(torch, vc))
            kv.set_length(0, n0)
            o = torch.empty(nq * hd, device="cuda")
            if fused:
                kv.step(0, cu(torch, q), cu(torch, k), cu(torch, v), o, 1.0, n0, window,
                        cu(torch, qn), cu(torch, kn), True, 1e-6, cu(torch, freq))
            else:
                qr = torch.empty(nq * hd, device="cuda")
                kv.append_rope(0, cu(torch, q), cu(torch, k), cu(torch, v), qr, cu(torch, qn),
                               cu(torch, kn), True, 1e-6, cu(torch, freq), n0)
                kv.decode(0, qr, o, 1.0, n0, window)
            kv.check()
            kt, vt = kv.layer_tensors(0)
            outs.append((o.cpu().numpy(), kt[:, :n0 + 1].cpu().numpy(),
                         vt[:, :n0 + 1].cpu().numpy()))
        finally:
            kv.close()
    for a, b in zip(outs[0], outs[1]):
        assert np.array_equal(a, b)
    # oracle: forward.h's prologue, the new row quantized into the cache
    qr = np.concatenate([orc.rope_apply(orc.rmsnorm(q[h * hd:(h + 1) * hd], qn, 1e-6), hd, n0,
                                        freq) for h in range(nq)])
    knew = np.concatenate([orc.rope_apply(orc.rmsnorm(k[h * hd:(h + 1) * hd], kn, 1e-6), hd, n0,
                                          freq) for h in range(nkv)])
    vnew = orc.rmsnorm_plain(v, 1e-6)
    K = np.vstack([kc, knew[None]])
    V = np.vstack([vc, vnew[None]])
    for raw, rows in ((outs[0][1], K), (outs[0][2], V)):
        got_q, got_s = mb.q8_unpack(raw.transpose(1, 0, 2), hd)
        wq, ws, _ = oracle_q8(orc, rows, nkv, hd)
        # rows written from the host: bit for bit
        assert np.array_equal(got_q[:n0], wq[:n0]) and np.array_equal(got_s[:n0], ws[:n0])
        # the new row is quantized from the kernel's own RMSNorm / RoPE
        # values, which may differ from the oracle's correctly rounded libm
        # by an ulp: its scales to a few ulps, its codes to at most one step
        assert np.max(np.abs(got_s[n0] - ws[n0]) / ws[n0]) <= 5e-7
        assert np.max(np.abs(got_q[n0].astype(np.int32) - wq[n0])) <= 1
    _, _, Kd = oracle_q8(orc, K, nkv, hd)
    _, _, Vd = oracle_q8(orc, V, nkv, hd)
    want = orc.attn_decode_gqa_cache(qr, Kd, Vd, nq, nkv, n0 + 1, hd, 1.0, n0, window)
    assert orc.rel_err(outs[0][0].reshape(nq, hd), want) <= PARITY_TOL


@pytest.mark.parametrize("nq,nkv,hd,M,window", [
    (32, 8, 128, 200, 0),   # Llama-shaped prompt
    (8, 4, 256, 150, 64),   # gemma SWA layer, head_dim 256
    (16, 2, 64, 100, 0),    # G = 8, head_dim 64
])
def test_prefill_on_q8_cache(mb, torch_cuda, orc, nq, nkv, hd, M, window):
    """The multi-token prologue writes Q8 rows; prefill attention reads them
    back (codes expanded per tile) and matches the reference's prefill on
    the dequantized cache; a decode after it reads the same rows."""
    torch = torch_cuda
    rng = np.random.default_rng(M + hd)
    q = rng.standard_normal((M, nq, hd)).astype(np.float32)
    k = rng.standard_normal((M, nkv, hd)).astype(np.float32)
    v = rng.standard_normal((M, nkv, hd)).astype(np.float32)
    kv = mb.KVCache(1, nkv, hd, M + 1, dtype="q8")
    try:
        qr = torch.empty((M, nq, hd), device="cuda")
        kv.append_rope_tokens(0, cu(torch, q), cu(torch, k), cu(torch, v), qr, pos0=0)
        kv.check()
        assert kv.length(0) == M
        assert_cache_equals(mb, orc, kv, 0, M, k.reshape(M, -1), v.reshape(M, -1))
        _, _, kd = oracle_q8(orc, k.reshape(M, -1), nkv, hd)
        _, _, vd = oracle_q8(orc, v.reshape(M, -1), nkv, hd)
        out = torch.full((M, nq, hd), float("nan"), device="cuda")
        kv.prefill(0, qr, out, hd ** -0.5, 0, window)
        kv.check()
        want = orc.attn_prefill_gqa(q, kd, vd, nq, nkv, M, M, hd, hd ** -0.5, 0, window)
        assert orc.rel_err(out.cpu().numpy(), want) <= PARITY_TOL
        o = torch.empty(nq * hd, device="cuda")
        kv.decode(0, qr[M - 1].reshape(-1).contiguous(), o, hd ** -0.5, M - 1, window)
        kv.check()
        want1 = orc.attn_decode_gqa_cache(q[M - 1].reshape(-1), kd, vd, nq, nkv, M, hd,
                                          hd ** -0.5, M - 1, window)
        assert orc.rel_err(o.cpu().numpy().reshape(nq, hd), want1) <= PARITY_TOL
    finally:
        kv.close()


def test_fused_q8_new_rows_code_count(mb, torch_cuda, orc):
    """The new rows of 48 consecutive fused steps on a Q8 cache: every code
    of K (QK-norm + RoPE) and V (V-norm) against the oracle's quantization
    of the reference prologue's rows.  The kernel's RMSNorm / RoPE values
    may differ from the oracle's correctly rounded libm by an ulp, which
    moves a code only when x/scale lands within an ulp of a rounding
    boundary: the count of such codes is bounded and none moves by more
    than one step."""
    torch = torch_cuda
    nq, nkv, hd, n0, steps = 32, 8, 128, 300, 48
    rng = np.random.default_rng(4848)
    kc = rng.standard_normal((n0, nkv * hd)).astype(np.float32)
    vc = rng.standard_normal((n0, nkv * hd)).astype(np.float32)
    qn = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    kn = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    freq = orc.rope_inv_freq(5e5, hd)
    ks = rng.standard_normal((steps, nkv * hd)).astype(np.float32)
    vs = rng.standard_normal((steps, nkv * hd)).astype(np.float32)
    qs = rng.standard_normal((steps, nq * hd)).astype(np.float32)
    kv = mb.KVCache(1, nkv, hd, n0 + steps, dtype="q8")
    try:
        kv.write(0, 0, cu(torch, kc), cu(torch, vc))
        kv.set_length(0, n0)
        o = torch.empty(nq * hd, device="cuda")
        dqn, dkn, dfreq = cu(torch, qn), cu(torch, kn), cu(torch, freq)
        for t in range(steps):
            kv.step(0, cu(torch, qs[t]), cu(torch, ks[t]), cu(torch, vs[t]), o, hd ** -0.5,
                    n0 + t, 0, dqn, dkn, True, 1e-6, dfreq)
        kv.check()
        assert kv.length(0) == n0 + steps
        kt, vt = kv.layer_tensors(0)
        got_k = cache_rows(mb, kt[:, n0:], steps, hd)
        got_v = cache_rows(mb, vt[:, n0:], steps, hd)
    finally:
        kv.close()
    want_k = np.stack([np.concatenate([
        orc.rope_apply(orc.rmsnorm(ks[t, h * hd:(h + 1) * hd], kn, 1e-6), hd, n0 + t, freq)
        for h in range(nkv)]) for t in range(steps)])
    want_v = np.stack([orc.rmsnorm_plain(vs[t], 1e-6) for t in range(steps)])
    total = moved = 0
    for (gq, gs), rows in ((got_k, want_k), (got_v, want_v)):
        wq, ws, _ = oracle_q8(orc, rows, nkv, hd)
        assert np.max(np.abs(gs - ws) / ws) <= 5e-7
        dq = np.abs(gq.astype(np.int32) - wq.astype(np.int32))
        assert dq.max() <= 1
        total += dq.size
        moved += int(np.count_nonzero(dq))
    assert total == 2 * steps * nkv * hd
    assert moved <= total // 1000, f"{moved} of {total} codes differ by one step"
