"""GPU parity of the per-token prologue (QK RMSNorm, V norm, NEOX RoPE, KV
append: forward.h:554-575) and of the KV-cache handle's layer step
(forward.h:554-590) against the oracle and the reference's golden vectors."""
import os

import numpy as np
import pytest

from conftest import PARITY_TOL

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def cu(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("d,nq,nkv,pos,theta", [(128, 32, 8, 16384, 5e5), (256, 8, 4, 32768, 1e6),
                                                (64, 4, 2, 7, 1e4), (128, 8, 1, 0, 1e4)])
@pytest.mark.parametrize("norms", [True, False])
def test_norm_rope_append(mb, torch_cuda, orc, d, nq, nkv, pos, theta, norms):
    torch = torch_cuda
    rng = np.random.default_rng(d + pos)
    q = rng.standard_normal(nq * d).astype(np.float32)
    k = rng.standard_normal(nkv * d).astype(np.float32)
    v = rng.standard_normal(nkv * d).astype(np.float32)
    qn = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32) if norms else None
    kn = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32) if norms else None
    freq = orc.rope_inv_freq(theta, d)
    cap, slot = 10, 6
    kc = torch.zeros((cap, nkv * d), device="cuda")
    vc = torch.zeros((cap, nkv * d), device="cuda")
    q_out = torch.empty(nq * d, device="cuda")
    mb.norm_rope_append(cu(torch, q), cu(torch, k), cu(torch, v), q_out,
                        None if qn is None else cu(torch, qn),
                        None if kn is None else cu(torch, kn), norms, 1e-6, cu(torch, freq), pos,
                        kc, vc, slot, nq, nkv, d)
    torch.cuda.synchronize()
    qh = q.reshape(nq, d).copy()
    kh = k.reshape(nkv, d).copy()
    for h in range(nq):
        x = orc.rmsnorm(qh[h], qn, 1e-6) if norms else qh[h]
        qh[h] = orc.rope_apply(x, d, pos, freq)
    for h in range(nkv):
        x = orc.rmsnorm(kh[h], kn, 1e-6) if norms else kh[h]
        kh[h] = orc.rope_apply(x, d, pos, freq)
    vv = orc.rmsnorm_plain(v, 1e-6) if norms else v
    assert orc.rel_err(q_out.cpu().numpy(), qh.reshape(-1)) < 1e-6
    kc_h, vc_h = kc.cpu().numpy(), vc.cpu().numpy()
    assert orc.rel_err(kc_h[slot], kh.reshape(-1)) < 1e-6
    assert orc.rel_err(vc_h[slot], vv) < 1e-6
    others = np.delete(np.arange(cap), slot)
    assert not np.any(kc_h[others]) and not np.any(vc_h[others])


def test_nope_layer_leaves_vectors_unrotated(mb, torch_cuda):
    """freq == null is NoPE (forward.h:556,566): q/k pass through."""
    torch = torch_cuda
    nq, nkv, d = 4, 2, 128
    q = torch.randn(nq * d, device="cuda")
    k = torch.randn(nkv * d, device="cuda")
    v = torch.randn(nkv * d, device="cuda")
    kc = torch.zeros((2, nkv * d), device="cuda")
    vc = torch.zeros((2, nkv * d), device="cuda")
    q_out = torch.empty_like(q)
    mb.norm_rope_append(q, k, v, q_out, None, None, False, 1e-6, None, 99, kc, vc, 1, nq, nkv, d)
    torch.cuda.synchronize()
    assert torch.equal(q_out, q) and torch.equal(kc[1], k) and torch.equal(vc[1], v)


def test_layer_step_against_reference_golden(mb, torch_cuda, orc):
    """forward.h:554-590 through the KV handle vs the reference's own output."""
    torch = torch_cuda
    z = np.load(os.path.join(GOLDEN, "layer_step.npz"))
    nq, nkv, hd, n0, cap, window = (int(x) for x in z["params"])
    kv = mb.KVCache(1, nkv, hd, cap)
    try:
        kv.write(0, 0, cu(torch, z["kc"][:n0]), cu(torch, z["vc"][:n0]))
        kv.set_length(0, n0)
        q_rot = torch.empty(nq * hd, device="cuda")
        out = torch.empty(nq * hd, device="cuda")
        kv.append_rope(0, cu(torch, z["q"]), cu(torch, z["k"]), cu(torch, z["v"]), q_rot,
                       cu(torch, z["q_norm"]), cu(torch, z["k_norm"]), True, 1e-6,
                       cu(torch, z["freq"]), n0)
        assert kv.length(0) == n0 + 1
        kv.decode(0, q_rot, out, 1.0, n0, window)
        kv.check()
        kt, vt = kv.layer_tensors(0)
        assert orc.rel_err(q_rot.cpu().numpy(), z["q_rot"]) < 1e-6
        assert orc.rel_err(kt[:, n0].reshape(-1).cpu().numpy(), z["k_row"]) < 1e-6
        assert orc.rel_err(vt[:, n0].reshape(-1).cpu().numpy(), z["v_row"]) < 1e-6
        # the rows written by molot_kv_write land head-major
        kc = z["kc"][:n0].reshape(n0, nkv, hd).transpose(1, 0, 2)
        assert np.array_equal(kt[:, :n0].cpu().numpy(), kc)
        assert orc.rel_err(out.cpu().numpy().reshape(nq, hd), z["out"]) <= PARITY_TOL
    finally:
        kv.close()


def test_multi_token_decode_loop_and_shared_kv(mb, torch_cuda, orc):
    """Token-by-token decode through the handle over a 2-layer model where
    layer 1 shares layer 0's cache (model.h:565-583, forward.h:578-586)."""
    torch = torch_cuda
    nq, nkv, hd, cap = 8, 2, 128, 64
    rng = np.random.default_rng(5)
    freq = orc.rope_inv_freq(1e4, hd)
    kc = np.zeros((cap, nkv * hd), np.float32)
    vc = np.zeros_like(kc)
    n_host = 0
    kv = mb.KVCache(2, nkv, hd, cap)
    try:
        for pos in range(20):
            q = rng.standard_normal(nq * hd).astype(np.float32)
            k = rng.standard_normal(nkv * hd).astype(np.float32)
            v = rng.standard_normal(nkv * hd).astype(np.float32)
            q_rot = torch.empty(nq * hd, device="cuda")
            o0 = torch.empty(nq * hd, device="cuda")
            o1 = torch.empty(nq * hd, device="cuda")
            kv.append_rope(0, cu(torch, q), cu(torch, k), cu(torch, v), q_rot, None, None, False,
                           1e-6, cu(torch, freq), pos)
            kv.decode(0, q_rot, o0, hd ** -0.5, pos, 0)
            kv.decode(0, q_rot, o1, hd ** -0.5, pos, 8)  # shared-KV SWA reader of layer 0
            kv.check()
            q2 = q.copy()
            st, n_host, want0 = orc.attn_layer_step(q2, k.copy(), v.copy(), None, None, 0, 1e-6,
                                                    freq, pos, kc, vc, n_host, (nq, hd), nq, nkv,
                                                    hd, hd ** -0.5, 0)
            want1 = orc.attn_decode_gqa_cache(q2, kc, vc, nq, nkv, n_host, hd, hd ** -0.5, pos, 8)
            assert orc.rel_err(o0.cpu().numpy().reshape(nq, hd), want0) <= PARITY_TOL
            assert orc.rel_err(o1.cpu().numpy().reshape(nq, hd), want1) <= PARITY_TOL
        assert kv.length(0) == 20 and kv.length(1) == 0
    finally:
        kv.close()


def test_cache_full_and_empty_errors(mb, torch_cuda):
    torch = torch_cuda
    nq, nkv, hd = 4, 2, 64
    kv = mb.KVCache(2, nkv, hd, 1)
    try:
        q = torch.randn(nq * hd, device="cuda")
        k = torch.randn(nkv * hd, device="cuda")
        qo = torch.empty_like(q)
        kv.append_rope(0, q, k, k, qo, None, None, False, 1e-6, None, 0)
        with pytest.raises(mb.MolotError) as ei:
            kv.append_rope(0, q, k, k, qo, None, None, False, 1e-6, None, 1)
        assert ei.value.status == mb.ERR_CACHE_FULL
        with pytest.raises(mb.MolotError) as ei:
            kv.decode(1, qo, qo, 1.0, 0, 0)
        assert ei.value.status == mb.ERR_CACHE_EMPTY
        kv.check()
    finally:
        kv.close()


def test_q_only_rotation(mb, torch_cuda, orc):
    """molot_norm_rope_append_dev with k, v and the cache NULL: a shared-KV
    layer's query (forward.h:554-558) alone."""
    torch = torch_cuda
    nq, d, pos = 8, 256, 4321
    rng = np.random.default_rng(5)
    q = rng.standard_normal(nq * d).astype(np.float32)
    qn = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32)
    freq = orc.rope_inv_freq(1e6, d)
    q_out = torch.empty(nq * d, device="cuda")
    mb.norm_rope_append(cu(torch, q), None, None, q_out, cu(torch, qn), None, False, 1e-6,
                        cu(torch, freq), pos, None, None, 0, nq, 1, d)
    torch.cuda.synchronize()
    want = np.concatenate([orc.rope_apply(orc.rmsnorm(q[h * d:(h + 1) * d], qn, 1e-6), d, pos, freq)
                           for h in range(nq)])
    assert orc.rel_err(q_out.cpu().numpy(), want) < 1e-6
    with pytest.raises(mb.MolotError):  # k given without its cache
        mb.norm_rope_append(cu(torch, q), cu(torch, q[:d]), None, q_out, None, None, False, 1e-6,
                            None, pos, None, None, 0, nq, 1, d)
