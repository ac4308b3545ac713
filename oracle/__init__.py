"""TEST INFRASTRUCTURE ONLY: CPU checkers for the molot_b200 kernels.

Two checkers live here, both plain host code:

* ``port`` -- ``attn_oracle.c``, a C restatement of the reference path
  (include/molot/attn.h, norm.h, gemm.h, forward.h:554-590), built into
  ``oracle/_build/libmolot_oracle.so``.
* ``ref``  -- the reference's own headers compiled unchanged behind the C ABI
  of ``ref_shim.cc``, built into ``oracle/_ref/libmolot_ref.so`` when the
  reference tree is present at build time (the built file then travels with
  the repository snapshot).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg import this package, and only as the checker or the timed CPU baseline.
The product library (``molot_b200``) never imports, links or calls it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PORT_SO = os.path.join(HERE, "_build", "libmolot_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libmolot_ref.so")


def _reference_tree() -> str | None:
    """Root of the reference's source tree: MOLOT_REFERENCE_TREE, else the
    reference_path that BASELINE.json records for this repository; None
    when neither names an existing tree (then only the port is built and
    ref() is None)."""
    cand = os.environ.get("MOLOT_REFERENCE_TREE")
    if not cand:
        try:
            import json
            with open(os.path.join(os.path.dirname(HERE), "BASELINE.json")) as fh:
                cand = json.load(fh).get("reference_path")
        except (OSError, ValueError):
            cand = None
    if cand and os.path.isfile(os.path.join(cand, "include", "molot", "attn.h")):
        return cand
    return None


REF_TREE = _reference_tree()


def require_reference_tree() -> str:
    """The reference tree, or a clear error naming how to point at it."""
    if REF_TREE is None:
        raise RuntimeError("reference source tree not found: set MOLOT_REFERENCE_TREE to the "
                           "directory holding include/molot/attn.h")
    return REF_TREE

_f = ctypes.c_float
_i = ctypes.c_int
_p = ctypes.c_void_p

_port = None
_ref = None
_ref_checked = False

_AVX512_FLAGS = ("avx512f", "avx512bw", "avx512dq", "avx512vl", "avx512cd")


def build(with_ref: bool | None = None) -> None:
    """Compile the C restatement, and the reference shim when the reference
    tree exists (``with_ref=None``) or when asked to (``with_ref=True``)."""
    env = dict(os.environ)
    # The image's default CC/CXX wrapper is fine for both targets; make them
    # explicit so a stray environment cannot change the flags' meaning.
    targets = ["port"]
    cmd = ["make", "-s", "-C", HERE]
    if with_ref or (with_ref is None and REF_TREE is not None):
        targets.append("ref")
        cmd.append(f"REF={require_reference_tree()}")
    subprocess.run(cmd + targets, check=True, env=env)


def host_has_avx512() -> bool:
    try:
        with open("/proc/cpuinfo") as fh:
            for line in fh:
                if line.startswith("flags"):
                    flags = set(line.split(":", 1)[1].split())
                    return all(f in flags for f in _AVX512_FLAGS)
    except OSError:
        pass
    return False


def _declare(lib, name, argtypes, restype=None):
    fn = getattr(lib, name)
    fn.argtypes = argtypes
    fn.restype = restype
    return fn


def port():
    """The C restatement (always available once built)."""
    global _port
    if _port is None:
        if not os.path.isfile(PORT_SO):
            build(with_ref=False)
        lib = ctypes.CDLL(PORT_SO)
        _declare(lib, "oracle_dot", [_p, _p, _i], _f)
        _declare(lib, "oracle_exp_taylor", [_f], _f)
        _declare(lib, "oracle_rope_apply", [_p, _i, _i, _p])
        _declare(lib, "oracle_rope_inv_freq", [_f, _i, _p])
        _declare(lib, "oracle_rmsnorm", [_p, _p, _p, _i, _f])
        _declare(lib, "oracle_rmsnorm_plain", [_p, _p, _i, _f])
        _declare(lib, "oracle_attn_decode_gqa_cache", [_p, _p, _p, _p, _i, _i, _i, _i, _f, _i, _i])
        _declare(lib, "oracle_attn_decode_gqa_win", [_p, _p, _p, _p, _i, _i, _i, _i, _f, _i, _i])
        _declare(lib, "oracle_attn_decode_gqa_cache_f64",
                 [_p, _p, _p, _p, _i, _i, _i, _i, ctypes.c_double, _i, _i])
        _declare(lib, "oracle_attn_layer_step",
                 [_p, _p, _p, _p, _p, _i, _f, _p, _i, _p, _p, _p, _i, _p, _i, _i, _i, _f, _i], _i)
        _declare(lib, "oracle_attn_decode_paged",
                 [_p, _p, _p, _p, _p, _i, _p, _p, _i, _i, _i, _i, _i, _f, _i])
        _declare(lib, "oracle_attn_prefill_gqa",
                 [_p, _p, _p, _p, _i, _i, _i, _i, _i, _f, _i, _i])
        _declare(lib, "oracle_quantize_q4", [_p, _i, _i, _p, _p, _p, _p])
        _declare(lib, "oracle_quantize_act_q8", [_p, _i, _p, _p])
        _declare(lib, "oracle_quantize_q8_blocks", [_p, ctypes.c_long, _p, _p])
        _declare(lib, "oracle_gemv_q4", [_p, _p, _p, _i, _i, _p, _p])
        _port = lib
    return _port


def ref():
    """The reference's own attn.h behind ref_shim.cc, or None when it was not
    built or this host cannot execute AVX-512."""
    global _ref, _ref_checked
    if not _ref_checked:
        _ref_checked = True
        if os.path.isfile(PORT_SO) and not os.path.isfile(REF_SO) and REF_TREE is not None:
            try:
                build(with_ref=True)
            except subprocess.CalledProcessError:
                pass
        if os.path.isfile(REF_SO) and host_has_avx512():
            lib = ctypes.CDLL(REF_SO)
            _declare(lib, "ref_pool_size", [_i], _i)
            _declare(lib, "ref_attn_decode_gqa_cache", [_p, _p, _p, _p, _i, _i, _i, _i, _f, _i, _i, _i])
            _declare(lib, "ref_attn_decode_gqa", [_p, _p, _p, _p, _i, _i, _i, _i, _f, _i])
            _declare(lib, "ref_attn_decode_gqa_win", [_p, _p, _p, _p, _i, _i, _i, _i, _f, _i, _i, _i])
            _declare(lib, "ref_attn_decode_head_win", [_p, _p, _p, _p, _i, _i, _f, _i, _i])
            _declare(lib, "ref_attn_decode_head", [_p, _p, _p, _p, _i, _i, _f])
            _declare(lib, "ref_rope_apply", [_p, _i, _i, _p])
            _declare(lib, "ref_rope_inv_freq", [_f, _i, _p])
            _declare(lib, "ref_rmsnorm", [_p, _p, _p, _i, _f])
            _declare(lib, "ref_rmsnorm_plain", [_p, _p, _i, _f])
            _declare(lib, "ref_exp16", [_p, _p])
            _declare(lib, "ref_dot", [_p, _p, _i], _f)
            _declare(lib, "ref_attn_layer_step",
                     [_p, _p, _p, _p, _p, _i, _f, _p, _i, _p, _p, _p, _i, _p, _i, _i, _i, _f, _i, _i], _i)
            for name, args in (("ref_quantize_q4", [_p, _i, _i, _p, _p, _p, _p]),
                               ("ref_quantize_act_q8", [_p, _i, _p, _p]),
                               ("ref_quantize_q8_blocks", [_p, ctypes.c_long, _p, _p]),
                               ("ref_gemv_q4", [_p, _p, _p, _p, _i, _i, _p, _p, _i])):
                if hasattr(lib, name):
                    _declare(lib, name, args)
            if hasattr(lib, "ref_attn_prefill_gqa"):
                _declare(lib, "ref_attn_prefill_gqa",
                         [_p, _p, _p, _p, _i, _i, _i, _i, _i, _f, _i, _i, _i])
            _ref = lib
    return _ref


def _ptr(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "oracle inputs must be C-contiguous"
    return a.ctypes.data


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


# ---------------------------------------------------------------- wrappers

def attn_decode_gqa_cache(Q, K, V, nq, nkv, n, qhd, scale, pos_cur, window, impl="port",
                          nthreads=0):
    """attn.h:125-177 on host arrays: Q [nq*qhd], K/V [n][nkv*qhd]."""
    Q, K, V = _f32(Q), _f32(K), _f32(V)
    O = np.zeros((nq, qhd), np.float32)
    if impl == "port":
        port().oracle_attn_decode_gqa_cache(_ptr(Q), _ptr(K), _ptr(V), _ptr(O), nq, nkv, n, qhd,
                                            scale, pos_cur, window)
    elif impl == "ref":
        lib = ref()
        if lib is None:
            raise RuntimeError("reference shim unavailable on this host")
        lib.ref_attn_decode_gqa_cache(_ptr(Q), _ptr(K), _ptr(V), _ptr(O), nq, nkv, n, qhd, scale,
                                      pos_cur, window, nthreads or (os.cpu_count() or 1))
    else:
        raise ValueError(impl)
    return O


def attn_decode_gqa_cache_f64(Q, K, V, nq, nkv, n, qhd, scale, pos_cur, window):
    Q, K, V = _f32(Q), _f32(K), _f32(V)
    O = np.zeros((nq, qhd), np.float64)
    port().oracle_attn_decode_gqa_cache_f64(_ptr(Q), _ptr(K), _ptr(V), _ptr(O), nq, nkv, n, qhd,
                                            float(scale), pos_cur, window)
    return O


def attn_decode_gqa_win(Q, K, V, nq, nkv, n, d, scale, pos_cur, window, impl="port",
                        nthreads=0):
    """attn.h:178-187 on host arrays: K/V [nkv][n][d]."""
    Q, K, V = _f32(Q), _f32(K), _f32(V)
    O = np.zeros((nq, d), np.float32)
    if impl == "port":
        port().oracle_attn_decode_gqa_win(_ptr(Q), _ptr(K), _ptr(V), _ptr(O), nq, nkv, n, d,
                                          scale, pos_cur, window)
    else:
        lib = ref()
        if lib is None:
            raise RuntimeError("reference shim unavailable on this host")
        lib.ref_attn_decode_gqa_win(_ptr(Q), _ptr(K), _ptr(V), _ptr(O), nq, nkv, n, d, scale,
                                    pos_cur, window, nthreads or (os.cpu_count() or 1))
    return O


def attn_decode_paged(Q, Kpool, Vpool, block_table, seq_lens, positions, B, nq, nkv, d,
                      page_size, scale, window):
    """Per-sequence gather of a [page][nkv][page_size][d] pool, then attn.h:125-177."""
    Q, Kpool, Vpool = _f32(Q), _f32(Kpool), _f32(Vpool)
    bt = np.ascontiguousarray(block_table, dtype=np.int32)
    sl = np.ascontiguousarray(seq_lens, dtype=np.int32)
    pos = None if positions is None else np.ascontiguousarray(positions, dtype=np.int32)
    O = np.zeros((B, nq, d), np.float32)
    port().oracle_attn_decode_paged(_ptr(Q), _ptr(Kpool), _ptr(Vpool), _ptr(O), _ptr(bt),
                                    bt.shape[1], _ptr(sl), _ptr(pos), B, nq, nkv, d, page_size,
                                    scale, window)
    return O


def attn_layer_step(q, k, v, q_norm, k_norm, v_norm, eps, freq, pos, kc, vc, n, out_shape,
                    nq, nkv, hd, scale, window, impl="port", nthreads=0):
    """forward.h:554-590 for one layer; q/k/v/kc/vc are modified in place.
    Returns (status, new_n, out)."""
    cap = kc.shape[0]
    nn = ctypes.c_int(n)
    out = np.zeros(out_shape, np.float32)
    args = [_ptr(q), _ptr(k), _ptr(v), _ptr(q_norm), _ptr(k_norm), int(v_norm), eps, _ptr(freq),
            pos, _ptr(kc), _ptr(vc), ctypes.addressof(nn), cap, _ptr(out), nq, nkv, hd, scale,
            window]
    if impl == "port":
        st = port().oracle_attn_layer_step(*args)
    else:
        lib = ref()
        if lib is None:
            raise RuntimeError("reference shim unavailable on this host")
        st = lib.ref_attn_layer_step(*args, nthreads or (os.cpu_count() or 1))
    return st, nn.value, out


def attn_prefill_gqa(Qm, K, V, nq, nkv, M, N, d, scale, pos0, window, impl="port",
                     nthreads=0):
    """gemm.h:409-446 on host arrays: Qm [M][nq][d], K/V [N][nkv*d] (at least
    N rows); returns Om [M][nq][d]."""
    Qm, K, V = _f32(Qm), _f32(K), _f32(V)
    Om = np.zeros((M, nq, d), np.float32)
    if impl == "port":
        port().oracle_attn_prefill_gqa(_ptr(Qm), _ptr(K), _ptr(V), _ptr(Om), nq, nkv, M, N, d,
                                       scale, pos0, window)
    else:
        lib = ref()
        if lib is None:
            raise RuntimeError("reference shim unavailable on this host")
        lib.ref_attn_prefill_gqa(_ptr(Qm), _ptr(K), _ptr(V), _ptr(Om), nq, nkv, M, N, d, scale,
                                 pos0, window, nthreads or (os.cpu_count() or 1))
    return Om


def quantize_q4(W, impl="port"):
    """quant.h:112-123: FP32 [rows][cols] -> (scales f32 [rows][ng], zeros i8,
    data u8 [rows][cols/2], wsums i16), ng = cols/32."""
    W = _f32(W)
    rows, cols = W.shape
    ng = cols // 32
    sc = np.zeros((rows, ng), np.float32)
    z = np.zeros((rows, ng), np.int8)
    data = np.zeros((rows, cols // 2), np.uint8)
    ws = np.zeros((rows, ng), np.int16)
    fn = port().oracle_quantize_q4 if impl == "port" else ref().ref_quantize_q4
    fn(_ptr(W), rows, cols, _ptr(sc), _ptr(z), _ptr(data), _ptr(ws))
    return sc, z, data, ws


def quantize_act_q8(x, impl="port"):
    """gemm.h:44-70: x [n] -> (q i8 [n], scales f32 [ceil(n/32)])."""
    x = _f32(x)
    q = np.zeros(x.size, np.int8)
    sc = np.zeros((x.size + 31) // 32, np.float32)
    fn = port().oracle_quantize_act_q8 if impl == "port" else ref().ref_quantize_act_q8
    fn(_ptr(x), x.size, _ptr(q), _ptr(sc))
    return q, sc


def quantize_q8_blocks(x, impl="port"):
    """quant.h:33-43 per 32-value block (the Q8 KV row rule): x [..., m*32]
    -> (codes int8 [..., m*32], scales float32 [..., m])."""
    x = _f32(x)
    q = np.zeros(x.shape, np.int8)
    sc = np.zeros(x.shape[:-1] + (x.shape[-1] // 32,), np.float32)
    fn = port().oracle_quantize_q8_blocks if impl == "port" else ref().ref_quantize_q8_blocks
    fn(_ptr(x), x.size, _ptr(q), _ptr(sc))
    return q, sc


def dequantize_q8_blocks(q, sc):
    """Codes and per-32 scales back to float32: (float)q * s, one rounding."""
    q = np.asarray(q, np.int8)
    s = np.repeat(np.asarray(sc, np.float32), 32, axis=-1)
    return (q.astype(np.float32) * s).astype(np.float32)


def gemv_q4(q4, x, impl="port", nthreads=0):
    """gemm.h:223-254: y = W x for a Q4 matrix from quantize_q4."""
    sc, z, data, ws = q4
    rows, ng = sc.shape
    cols = ng * 32
    x = _f32(x)
    y = np.zeros(rows, np.float32)
    if impl == "port":
        port().oracle_gemv_q4(_ptr(sc), _ptr(z), _ptr(data), rows, cols, _ptr(x), _ptr(y))
    else:
        ref().ref_gemv_q4(_ptr(sc), _ptr(z), _ptr(data), _ptr(ws), rows, cols, _ptr(x), _ptr(y),
                          nthreads or (os.cpu_count() or 1))
    return y


def rope_apply(x, d, pos, inv_freq, impl="port"):
    x = _f32(x).copy()
    f = _f32(inv_freq)
    lib = port() if impl == "port" else ref()
    fn = lib.oracle_rope_apply if impl == "port" else lib.ref_rope_apply
    for h in range(x.size // d):
        fn(x.ctypes.data + 4 * h * d, d, pos, _ptr(f))
    return x


def rope_inv_freq(base, d, impl="port"):
    out = np.zeros(d // 2, np.float32)
    if impl == "port":
        port().oracle_rope_inv_freq(base, d, _ptr(out))
    else:
        ref().ref_rope_inv_freq(base, d, _ptr(out))
    return out


def rmsnorm(x, w, eps, impl="port"):
    x, w = _f32(x), _f32(w)
    y = np.zeros_like(x)
    if impl == "port":
        port().oracle_rmsnorm(_ptr(x), _ptr(w), _ptr(y), x.size, eps)
    else:
        ref().ref_rmsnorm(_ptr(x), _ptr(w), _ptr(y), x.size, eps)
    return y


def rmsnorm_plain(x, eps, impl="port"):
    x = _f32(x)
    y = np.zeros_like(x)
    if impl == "port":
        port().oracle_rmsnorm_plain(_ptr(x), _ptr(y), x.size, eps)
    else:
        ref().ref_rmsnorm_plain(_ptr(x), _ptr(y), x.size, eps)
    return y


def dot(a, b, impl="port"):
    a, b = _f32(a), _f32(b)
    if impl == "port":
        return port().oracle_dot(_ptr(a), _ptr(b), a.size)
    return ref().ref_dot(_ptr(a), _ptr(b), a.size)


def exp_taylor(x, impl="port"):
    x = _f32(x)
    if impl == "port":
        fn = port().oracle_exp_taylor
        return np.array([fn(float(v)) for v in x], np.float32)
    assert x.size == 16
    out = np.zeros(16, np.float32)
    ref().ref_exp16(_ptr(x), _ptr(out))
    return out


def rel_err(got, want) -> float:
    """max |got - want| / max |want|: the parity metric of the path."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    denom = float(np.max(np.abs(want))) if want.size else 0.0
    if denom == 0.0:
        return float(np.max(np.abs(got))) if got.size else 0.0
    return float(np.max(np.abs(got - want)) / denom)
