"""molot_attn_step: forward.h:554-590 (QK-norm, V-norm, RoPE, KV append and
decode attention) in one launch, against the reference's golden vectors,
the oracle, and the two-launch path (append + decode) it replaces."""
import os

import numpy as np
import pytest

from conftest import PARITY_TOL

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def cu(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def test_step_against_reference_golden(mb, torch_cuda, orc):
    torch = torch_cuda
    z = np.load(os.path.join(GOLDEN, "layer_step.npz"))
    nq, nkv, hd, n0, cap, window = (int(x) for x in z["params"])
    kv = mb.KVCache(1, nkv, hd, cap)
    try:
        kv.write(0, 0, cu(torch, z["kc"][:n0]), cu(torch, z["vc"][:n0]))
        kv.set_length(0, n0)
        out = torch.empty(nq * hd, device="cuda")
        kv.step(0, cu(torch, z["q"]), cu(torch, z["k"]), cu(torch, z["v"]), out, 1.0, n0, window,
                cu(torch, z["q_norm"]), cu(torch, z["k_norm"]), True, 1e-6, cu(torch, z["freq"]))
        kv.check()
        assert kv.length(0) == n0 + 1
        kt, vt = kv.layer_tensors(0)
        assert orc.rel_err(kt[:, n0].reshape(-1).cpu().numpy(), z["k_row"]) < 1e-6
        assert orc.rel_err(vt[:, n0].reshape(-1).cpu().numpy(), z["v_row"]) < 1e-6
        assert orc.rel_err(out.cpu().numpy().reshape(nq, hd), z["out"]) <= PARITY_TOL
    finally:
        kv.close()


@pytest.mark.parametrize("nq,nkv,hd,n0,norms,window", [
    (32, 8, 128, 4096, True, 0),      # cfg1 shape
    (32, 8, 128, 16384, False, 0),    # cfg2 shape, no QK-norm
    (8, 4, 256, 2000, True, 1024),    # gemma SWA layer
    (16, 2, 64, 63, True, 0),         # new slot 63 closes a 64-slot tile
    (16, 2, 64, 64, False, 0),        # new slot opens a tile
    (8, 1, 128, 15, True, 0),         # new slot closes a 16-slot block
    (4, 4, 128, 0, True, 0),          # first token: the new row is all there is
    (32, 8, 128, 300, True, 0),       # ~1 block per CTA: the shortened last share
    (64, 8, 128, 2500, False, 0),     # G = 8
    (8, 8, 128, 40000, True, 0),      # G = 1, long
    # long enough for the split-barrier kernels
    (64, 8, 128, 20000, True, 0),     # G = 8: two head sets
    (32, 8, 64, 40000, False, 0),     # head_dim 64
    (32, 8, 128, 30000, True, 20000), # window start inside a tile
])
def test_step_matches_oracle_and_two_launch_path(mb, torch_cuda, orc, nq, nkv, hd, n0, norms,
                                                  window):
    torch = torch_cuda
    rng = np.random.default_rng(n0 + hd)
    cap = n0 + 4
    kc = np.zeros((cap, nkv * hd), np.float32)
    vc = np.zeros_like(kc)
    kc[:n0] = rng.standard_normal((n0, nkv * hd))
    vc[:n0] = rng.standard_normal((n0, nkv * hd))
    q = rng.standard_normal(nq * hd).astype(np.float32)
    k = rng.standard_normal(nkv * hd).astype(np.float32)
    v = rng.standard_normal(nkv * hd).astype(np.float32)
    qn = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32) if norms else None
    kn = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32) if norms else None
    freq = orc.rope_inv_freq(5e5, hd)
    scale = hd ** -0.5
    outs = []
    for fused in (True, False):
        kv = mb.KVCache(1, nkv, hd, cap)
        try:
            if n0:
                kv.write(0, 0, cu(torch, kc[:n0]), cu(torch, vc[:n0]))
            kv.set_length(0, n0)
            out = torch.empty(nq * hd, device="cuda")
            dqn = None if qn is None else cu(torch, qn)
            dkn = None if kn is None else cu(torch, kn)
            if fused:
                kv.step(0, cu(torch, q), cu(torch, k), cu(torch, v), out, scale, n0, window, dqn,
                        dkn, norms, 1e-6, cu(torch, freq))
            else:
                q_rot = torch.empty(nq * hd, device="cuda")
                kv.append_rope(0, cu(torch, q), cu(torch, k), cu(torch, v), q_rot, dqn, dkn,
                               norms, 1e-6, cu(torch, freq), n0)
                kv.decode(0, q_rot, out, scale, n0, window)
            kv.check()
            kt, vt = kv.layer_tensors(0)
            outs.append((out.cpu().numpy().reshape(nq, hd), kt[:, n0].cpu().numpy(),
                         vt[:, n0].cpu().numpy()))
        finally:
            kv.close()
    # one launch == two launches, bit for bit (same arithmetic, same split)
    for a, b in zip(outs[0], outs[1]):
        assert np.array_equal(a.view(np.int32), b.view(np.int32))
    st, n1, want = orc.attn_layer_step(q.copy(), k.copy(), v.copy(), qn, kn, int(norms), 1e-6, freq,
                                       n0, kc, vc, n0, (nq, hd), nq, nkv, hd, scale, window)
    assert st == 0 and n1 == n0 + 1
    assert orc.rel_err(outs[0][0], want) <= PARITY_TOL
    assert orc.rel_err(outs[0][1].reshape(-1), kc[n0]) < 1e-6


def test_step_token_loop_with_shared_reader(mb, torch_cuda, orc):
    """40 tokens through step() on layer 0, each followed by a shared-KV
    window reader of layer 0 (model.h:565-583), against the oracle."""
    torch = torch_cuda
    nq, nkv, hd, cap = 8, 2, 128, 64
    rng = np.random.default_rng(9)
    freq = orc.rope_inv_freq(1e4, hd)
    kc = np.zeros((cap, nkv * hd), np.float32)
    vc = np.zeros_like(kc)
    n_host = 0
    kv = mb.KVCache(2, nkv, hd, cap)
    try:
        for pos in range(40):
            q = rng.standard_normal(nq * hd).astype(np.float32)
            k = rng.standard_normal(nkv * hd).astype(np.float32)
            v = rng.standard_normal(nkv * hd).astype(np.float32)
            o0 = torch.empty(nq * hd, device="cuda")
            o1 = torch.empty(nq * hd, device="cuda")
            kv.step(0, cu(torch, q), cu(torch, k), cu(torch, v), o0, hd ** -0.5, pos, 0,
                    freq=cu(torch, freq))
            q_rot = torch.from_numpy(orc.rope_apply(q, hd, pos, freq)).cuda()
            kv.decode(0, q_rot, o1, hd ** -0.5, pos, 8)
            kv.check()
            q2 = q.copy()
            st, n_host, want0 = orc.attn_layer_step(q2, k.copy(), v.copy(), None, None, 0, 1e-6,
                                                    freq, pos, kc, vc, n_host, (nq, hd), nq, nkv,
                                                    hd, hd ** -0.5, 0)
            want1 = orc.attn_decode_gqa_cache(q2, kc, vc, nq, nkv, n_host, hd, hd ** -0.5, pos, 8)
            assert orc.rel_err(o0.cpu().numpy().reshape(nq, hd), want0) <= PARITY_TOL, pos
            assert orc.rel_err(o1.cpu().numpy().reshape(nq, hd), want1) <= PARITY_TOL, pos
    finally:
        kv.close()


def test_step_cache_full(mb, torch_cuda):
    torch = torch_cuda
    kv = mb.KVCache(1, 1, 64, 1)
    try:
        x = torch.randn(64, device="cuda")
        o = torch.empty(64, device="cuda")
        kv.step(0, x, x, x, o, 1.0, 0)
        with pytest.raises(mb.MolotError) as ei:
            kv.step(0, x, x, x, o, 1.0, 1)
        assert ei.value.status == mb.ERR_CACHE_FULL
        kv.check()
    finally:
        kv.close()
