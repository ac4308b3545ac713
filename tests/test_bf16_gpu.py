"""BF16 KV-cache storage (MOLOT_KV_BF16): every row entering the cache is
rounded to bf16 (nearest even), the attention math stays FP32.  The parity
contract: the reference's own algorithm run on the same bf16-rounded cache
(the oracle on rounded K/V), within the same 1e-5 bar."""
import numpy as np
import pytest

from conftest import PARITY_TOL

pytestmark = pytest.mark.gpu


def bf16(x):
    """Round float32 values to bf16 (nearest even), returned as float32."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return r.astype(np.uint32).view(np.float32).reshape(np.shape(x))


def cu(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def slot_major(kt, n):
    """[nkv][cap][hd] cache view -> [n][nkv*hd] float32 numpy."""
    return kt[:, :n].float().permute(1, 0, 2).reshape(n, -1).cpu().numpy()


def test_write_rounds_rows(mb, torch_cuda):
    torch = torch_cuda
    rng = np.random.default_rng(1)
    nkv, hd, cap, n = 4, 128, 40, 33
    k = rng.standard_normal((n, nkv * hd)).astype(np.float32)
    v = rng.standard_normal((n, nkv * hd)).astype(np.float32)
    kv = mb.KVCache(2, nkv, hd, cap, dtype="bf16")
    try:
        kv.write(0, 3, k, v)                       # host rows
        kv.write(1, 0, cu(torch, k), cu(torch, v))  # device rows
        kv.check()
        for layer, s0 in ((0, 3), (1, 0)):
            kt, vt = kv.layer_tensors(layer)
            assert kt.dtype == torch.bfloat16
            got_k = kt[:, s0:s0 + n].float().permute(1, 0, 2).reshape(n, -1).cpu().numpy()
            got_v = vt[:, s0:s0 + n].float().permute(1, 0, 2).reshape(n, -1).cpu().numpy()
            assert np.array_equal(got_k, bf16(k)) and np.array_equal(got_v, bf16(v))
    finally:
        kv.close()


@pytest.mark.parametrize("nq,nkv,hd,n,window", [
    (32, 8, 128, 4097, 0),    # cfg1 shape
    (8, 4, 256, 3000, 1024),  # gemma SWA layer
    (64, 8, 64, 777, 0),      # G = 8, d = 64
    (4, 4, 128, 17, 0),       # G = 1, ragged
])
def test_decode_on_bf16_cache(mb, torch_cuda, orc, nq, nkv, hd, n, window):
    torch = torch_cuda
    rng = np.random.default_rng(n + hd)
    k = rng.standard_normal((n, nkv * hd)).astype(np.float32)
    v = rng.standard_normal((n, nkv * hd)).astype(np.float32)
    q = rng.standard_normal(nq * hd).astype(np.float32)
    kv = mb.KVCache(1, nkv, hd, n, dtype="bf16")
    try:
        kv.write(0, 0, cu(torch, k), cu(torch, v))
        kv.set_length(0, n)
        o = torch.empty(nq * hd, device="cuda")
        kv.decode(0, cu(torch, q), o, hd ** -0.5, n - 1, window)
        kv.check()
        want = orc.attn_decode_gqa_cache(q, bf16(k), bf16(v), nq, nkv, n, hd, hd ** -0.5, n - 1,
                                         window)
        assert orc.rel_err(o.cpu().numpy().reshape(nq, hd), want) <= PARITY_TOL
    finally:
        kv.close()


@pytest.mark.parametrize("nq,nkv,hd,n0,window", [(32, 8, 128, 5000, 0), (8, 4, 256, 900, 256),
                                                 (16, 2, 64, 63, 0)])
def test_fused_step_on_bf16_cache(mb, torch_cuda, orc, nq, nkv, hd, n0, window):
    torch = torch_cuda
    rng = np.random.default_rng(n0)
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
        kv = mb.KVCache(1, nkv, hd, cap, dtype="bf16")
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
            outs.append((o.cpu().numpy(), slot_major(kt, n0 + 1), slot_major(vt, n0 + 1)))
        finally:
            kv.close()
    for a, b in zip(outs[0], outs[1]):  # one launch == two launches, bit for bit
        assert np.array_equal(a, b)
    # oracle: forward.h's prologue, the new row rounded into the rounded cache
    qr = np.concatenate([orc.rope_apply(orc.rmsnorm(q[h * hd:(h + 1) * hd], qn, 1e-6), hd, n0,
                                        freq) for h in range(nq)])
    knew = np.concatenate([orc.rope_apply(orc.rmsnorm(k[h * hd:(h + 1) * hd], kn, 1e-6), hd, n0,
                                          freq) for h in range(nkv)])
    vnew = orc.rmsnorm_plain(v, 1e-6)
    K = np.vstack([bf16(kc), bf16(knew)[None]])
    V = np.vstack([bf16(vc), bf16(vnew)[None]])
    assert np.array_equal(outs[0][1], K) and np.array_equal(outs[0][2], V)
    want = orc.attn_decode_gqa_cache(qr, K, V, nq, nkv, n0 + 1, hd, 1.0, n0, window)
    assert orc.rel_err(outs[0][0].reshape(nq, hd), want) <= PARITY_TOL


def test_prefill_on_bf16_cache(mb, torch_cuda, orc):
    torch = torch_cuda
    nq, nkv, hd, M = 32, 8, 128, 200
    rng = np.random.default_rng(5)
    q = rng.standard_normal((M, nq, hd)).astype(np.float32)
    k = rng.standard_normal((M, nkv, hd)).astype(np.float32)
    v = rng.standard_normal((M, nkv, hd)).astype(np.float32)
    kv = mb.KVCache(1, nkv, hd, M, dtype="bf16")
    try:
        qr = torch.empty((M, nq, hd), device="cuda")
        out = torch.empty((M, nq, hd), device="cuda")
        kv.append_rope_tokens(0, cu(torch, q), cu(torch, k), cu(torch, v), qr, pos0=0)
        kv.prefill(0, qr, out, hd ** -0.5, 0)
        kv.check()
        kt, vt = kv.layer_tensors(0)
        K, V = slot_major(kt, M), slot_major(vt, M)
        assert np.array_equal(K, bf16(k.reshape(M, -1))) and np.array_equal(V, bf16(v.reshape(M, -1)))
        want = orc.attn_prefill_gqa(q, K, V, nq, nkv, M, M, hd, hd ** -0.5, 0, 0)
        assert orc.rel_err(out.cpu().numpy(), want) <= PARITY_TOL
    finally:
        kv.close()
