"""Generates the golden fixtures in this directory from the reference itself.

    python tests/golden/make_golden.py

Runs the reference's own decode-attention headers (compiled unchanged into
oracle/_ref/libmolot_ref.so by oracle/Makefile) on seeded N(0,1) inputs and
stores inputs and outputs as .npz files.  tests/test_oracle.py pins the C
restatement in oracle/attn_oracle.c against them; nothing at run time needs
the reference tree.

Cases follow the reference's own checks (bench/bench.cc:186-234: attention
head at n=512, d=128 with inputs scaled by 0.2; vector exp on 16 fixed
inputs) and the forward-path function attn_decode_gqa_cache at small sizes
covering GQA grouping, the sliding window, head_dim 64/128/256, scale 1 and
1/sqrt(d), plus the per-token prologue (QK RMSNorm, V norm, RoPE, append).
"""
from __future__ import annotations

import os
import sys

import zlib

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402

# (name, nq, nkv, n, d, scale, pos_cur, window, seed)
ATTN_CASES = [
    ("gqa4_n300_d128", 8, 2, 300, 128, 128 ** -0.5, 299, 0, 11),
    ("mha_n45_d64_win16", 4, 4, 45, 64, 0.125, 44, 16, 12),
    ("gqa2_n70_d256_scale1", 8, 4, 70, 256, 1.0, 69, 0, 13),
    ("gqa4_n33_d128_tail", 32, 8, 33, 128, 128 ** -0.5, 32, 0, 14),
    ("gqa8_n200_d128_win1", 8, 1, 200, 128, 128 ** -0.5, 199, 1, 15),
    ("gqa4_n17_d128_winbig", 4, 1, 17, 128, 0.3, 16, 1024, 16),
    ("empty_window", 4, 2, 10, 64, 0.125, 40, 8, 17),
]


def attn_cases():
    out = {}
    for name, nq, nkv, n, d, scale, pos, window, seed in ATTN_CASES:
        rng = np.random.default_rng(seed)
        Q = rng.standard_normal((nq, d)).astype(np.float32)
        K = rng.standard_normal((n, nkv * d)).astype(np.float32)
        V = rng.standard_normal((n, nkv * d)).astype(np.float32)
        O = oracle.attn_decode_gqa_cache(Q, K, V, nq, nkv, n, d, scale, pos, window, impl="ref",
                                         nthreads=4)
        out[name] = dict(Q=Q, K=K, V=V, O=O,
                         params=np.array([nq, nkv, n, d, pos, window], np.int64),
                         scale=np.float32(scale))
    return out


def head_case():
    """bench.cc:186-218 shape: one head, n=512, d=128, N(0,1)*0.2."""
    rng = np.random.default_rng(1234)
    n, d = 512, 128
    Q = (rng.standard_normal(d) * 0.2).astype(np.float32)
    K = (rng.standard_normal((n, d)) * 0.2).astype(np.float32)
    V = (rng.standard_normal((n, d)) * 0.2).astype(np.float32)
    lib = oracle.ref()
    O = np.zeros(d, np.float32)
    lib.ref_attn_decode_head(Q.ctypes.data, K.ctypes.data, V.ctypes.data, O.ctypes.data, n, d,
                             np.float32(1.0 / np.sqrt(d)))
    return dict(Q=Q, K=K, V=V, O=O)


def exp_case():
    """bench.cc:220-234 inputs."""
    x = np.array([-87.0, -20.0, -10.0, -5.0, -3.0, -2.0, -1.5, -1.0, -0.75, -0.5, -0.25, -0.1,
                  -0.01, 0.0, 1.0, 50.0], np.float32)
    return dict(x=x, y=oracle.exp_taylor(x, impl="ref"))


def norm_rope_case():
    rng = np.random.default_rng(21)
    out = {}
    for d, base, pos in ((128, 1e4, 4096), (128, 5e5, 16384), (256, 1e6, 32768), (64, 1e4, 7)):
        x = rng.standard_normal(d).astype(np.float32)
        w = rng.standard_normal(d).astype(np.float32)
        inv = oracle.rope_inv_freq(base, d, impl="ref")
        out[f"d{d}_pos{pos}"] = dict(
            x=x, w=w, inv_freq=inv, pos=np.int64(pos), base=np.float32(base),
            rmsnorm=oracle.rmsnorm(x, w, 1e-6, impl="ref"),
            rmsnorm_plain=oracle.rmsnorm_plain(x, 1e-6, impl="ref"),
            rope=oracle.rope_apply(x, d, pos, inv, impl="ref"))
    return out


def layer_step_case():
    """forward.h:554-590 for a gemma-style layer: QK-norm, V-norm, RoPE."""
    rng = np.random.default_rng(31)
    nq, nkv, hd, n0, cap = 8, 4, 256, 40, 48
    kc = np.zeros((cap, nkv * hd), np.float32)
    vc = np.zeros((cap, nkv * hd), np.float32)
    kc[:n0] = rng.standard_normal((n0, nkv * hd))
    vc[:n0] = rng.standard_normal((n0, nkv * hd))
    q = rng.standard_normal(nq * hd).astype(np.float32)
    k = rng.standard_normal(nkv * hd).astype(np.float32)
    v = rng.standard_normal(nkv * hd).astype(np.float32)
    qn = (1.0 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    kn = (1.0 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    freq = oracle.rope_inv_freq(1e4, hd, impl="ref")
    inputs = dict(q=q.copy(), k=k.copy(), v=v.copy(), kc=kc.copy(), vc=vc.copy(), q_norm=qn,
                  k_norm=kn, freq=freq)
    st, n1, out = oracle.attn_layer_step(q, k, v, qn, kn, 1, 1e-6, freq, n0, kc, vc, n0,
                                         (nq, hd), nq, nkv, hd, 1.0, 16, impl="ref", nthreads=4)
    assert st == 0 and n1 == n0 + 1
    return dict(**inputs, params=np.array([nq, nkv, hd, n0, cap, 16], np.int64),
                out=out, q_rot=q, k_row=kc[n0].copy(), v_row=vc[n0].copy())


def prefill_cases():
    """gemm.h:409-446 causal prefill over a filled cache (forward.h:396): the
    cache holds pos0 earlier slots plus the M new ones (N = pos0 + M)."""
    out = {}
    specs = {
        "g4_d64_full": (8, 2, 64, 40, 20, 0, 0.125),
        "g4_d64_swa16": (8, 2, 64, 40, 20, 16, 0.125),
        "g4_d128": (8, 2, 128, 20, 45, 0, 128 ** -0.5),
        "g2_d256_swa": (4, 2, 256, 16, 30, 24, 1.0),
        "g8_d128_pos0": (8, 1, 128, 17, 0, 0, 128 ** -0.5),
    }
    for name, (nq, nkv, d, M, pos0, window, scale) in specs.items():
        rng = np.random.default_rng(zlib.crc32(name.encode()))
        N = pos0 + M
        Q = rng.standard_normal((M, nq, d)).astype(np.float32)
        K = rng.standard_normal((N, nkv * d)).astype(np.float32)
        V = rng.standard_normal((N, nkv * d)).astype(np.float32)
        O = oracle.attn_prefill_gqa(Q, K, V, nq, nkv, M, N, d, scale, pos0, window, impl="ref",
                                    nthreads=4)
        out[name] = dict(Q=Q, K=K, V=V, O=O, params=np.array([nq, nkv, d, M, N, pos0, window],
                                                              np.int64),
                         scale=np.float32(scale))
    return out


def gemv_q4_cases():
    """quant.h:112-123 weight quantization, gemm.h:44-70 activation
    quantization and gemm.h:223-254 gemv_q4, all run by the reference."""
    rng = np.random.default_rng(77)
    out = {}
    W = (rng.standard_normal((16, 256)) * 0.05).astype(np.float32)
    W[3, 32:64] = 0.0  # a flat group: scale 1, zero 0
    sc, z, data, ws = oracle.quantize_q4(W, impl="ref")
    out["quant"] = dict(W=W, scales=sc, zeros=z, data=data, wsums=ws)
    x = (rng.standard_normal(2048) * rng.uniform(0.1, 20, 2048)).astype(np.float32)
    x[64:96] = 0.0  # an all-zero activation block
    q, xs = oracle.quantize_act_q8(x, impl="ref")
    out["act"] = dict(x=x, q=q, scales=xs)
    for name, (rows, cols) in (("gemv_a", (96, 1024)), ("gemv_b", (33, 4096))):
        Wm = (rng.standard_normal((rows, cols)) * 0.03).astype(np.float32)
        q4 = oracle.quantize_q4(Wm, impl="ref")
        xv = (rng.standard_normal(cols) * 2).astype(np.float32)
        xv[:32] *= 50.0  # an outlier block
        y = oracle.gemv_q4(q4, xv, impl="ref", nthreads=4)
        out[name] = dict(scales=q4[0], zeros=q4[1], data=q4[2], wsums=q4[3], x=xv, y=y)
    return out


def kv_q8_case():
    """quant.h:33-50 quantize_q8_row run by the reference on each 32-value
    block: the block rule of the Q8 KV rows.  Rows of head_dim 128 with
    mixed magnitudes and outliers, an all-zero block, and a block whose
    absmax is 127 (so x/s is x itself) holding exact half-integers, which
    pins the ties-to-even rounding."""
    rng = np.random.default_rng(88)
    x = (rng.standard_normal((96, 128)) * rng.uniform(1e-3, 30, (96, 1))).astype(np.float32)
    x[::9, 7] *= 40.0
    x[5, 32:64] = 0.0
    tie = np.array([127.0] + [k + 0.5 for k in range(-15, 15)] + [-126.5], np.float32)
    x[6, :32] = tie
    q, sc = oracle.quantize_q8_blocks(x, impl="ref")
    return dict(x=x, q=q, scales=sc)


def flatten(cases):
    flat = {}
    for name, case in cases.items():
        for k, v in case.items():
            flat[f"{name}/{k}"] = v
    return flat


FIXTURES = {
    "attn_gqa_cache.npz": lambda: flatten(attn_cases()),
    "attn_head_bench.npz": head_case,
    "exp16.npz": exp_case,
    "norm_rope.npz": lambda: flatten(norm_rope_case()),
    "layer_step.npz": layer_step_case,
    "prefill.npz": lambda: flatten(prefill_cases()),
    "gemv_q4.npz": lambda: flatten(gemv_q4_cases()),
    "kv_q8.npz": kv_q8_case,
}


def main(names=None):
    """Write the named fixtures (all when none are given)."""
    if oracle.ref() is None:
        raise SystemExit("reference shim not available (needs the reference tree and AVX-512)")
    for fname in names or sorted(FIXTURES):
        np.savez_compressed(os.path.join(HERE, fname), **FIXTURES[fname]())
        print(fname, os.path.getsize(os.path.join(HERE, fname)))


if __name__ == "__main__":
    main(sys.argv[1:])
