"""molot_b200: B200-native decode attention with the reference's attn.h API.

Python view of the C ABI in ``include/molot_b200.h`` (``libmolot_b200.so``,
built in-tree by ``python -m molot_b200.build``).  Names, argument meaning
and error behaviour mirror the reference's functions
(include/molot/attn.h, the attention segment of include/molot/forward.h):

* host drop-ins on numpy arrays, synchronous:
  ``attn_decode_gqa_cache``, ``attn_decode_gqa``, ``attn_decode_gqa_win``,
  ``attn_decode_head``, ``attn_decode_head_win``, ``rope_apply``,
  ``rope_inv_freq``;
* stream-ordered device forms on torch CUDA tensors:
  ``decode_strided``, ``norm_rope_append``;
* ``KVCache`` (forward.h's per-layer KVC, HBM-resident) with
  ``append_rope`` / ``decode``;
* ``PagedPlan`` for batched decode over 16-token pages;
* ``Comm``, the peer-gather group of kv-head-sharded decode over several
  GPUs (``PagedPlan.decode_gather``).

torch is used only to hold device memory and streams.  There is no CPU
fallback: importing this package fails loudly when the library is missing.
"""
from __future__ import annotations

import ctypes
import os
import re

import numpy as np

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libmolot_b200.so")
HEADER = os.path.join(os.path.dirname(PKG), "include", "molot_b200.h")

OK = 0
ERR_INVALID = -1
ERR_CUDA = -2
ERR_NOMEM = -3
ERR_CACHE_FULL = -4
ERR_CACHE_EMPTY = -5
ERR_UNSUPPORTED = -6
ERR_TIMEOUT = -7
ERR_NO_DEVICE = -8

KV_F32 = 0   # molot_kv_dtype: the reference's FP32 cache
KV_BF16 = 1  # BF16 storage (rounded on entry), FP32 math
KV_Q8 = 2    # int8 codes + per-32 FP32 scales per row, FP32 math
_KV_DTYPES = {"f32": KV_F32, "bf16": KV_BF16, "q8": KV_Q8}


def q8_row_bytes(hd: int) -> int:
    """Bytes of one Q8 cache row: hd int8 codes, hd/32 float32 scales,
    padded to a multiple of 16."""
    return (hd + hd // 8 + 15) & ~15


def q8_unpack(rows, hd: int):
    """Q8 cache rows (uint8 [..., q8_row_bytes(hd)], numpy) -> (codes int8
    [..., hd], scales float32 [..., hd/32]); values read back as
    codes * scales repeated over each 32-value block."""
    rows = np.ascontiguousarray(rows, dtype=np.uint8)
    codes = rows[..., :hd].view(np.int8)
    scales = np.ascontiguousarray(rows[..., hd:hd + hd // 8]).view(np.float32)
    return codes, scales


class MolotError(RuntimeError):
    """A non-zero status from the C ABI (the reference throws
    std::runtime_error in the same places, forward.h:570,580)."""

    def __init__(self, status: int, text: str, detail: str):
        super().__init__(f"molot_b200 status {status} ({text}): {detail}")
        self.status = status


if not os.path.isfile(LIB_PATH):
    raise ImportError(
        f"molot_b200: CUDA library not built ({LIB_PATH} missing); "
        "run `python -m molot_b200.build` -- there is no CPU fallback")

_lib = ctypes.CDLL(LIB_PATH)

_p = ctypes.c_void_p
_i = ctypes.c_int
_f = ctypes.c_float
_ll = ctypes.c_longlong
_pp = ctypes.POINTER(ctypes.c_void_p)


def _decl(name, args, res=_i):
    fn = getattr(_lib, name)
    fn.argtypes = args
    fn.restype = res
    return fn


_decl("molot_status_string", [_i], ctypes.c_char_p)
_decl("molot_last_error", [], ctypes.c_char_p)
_decl("molot_device_status", [_i])
_decl("molot_attn_decode_gqa_cache", [_p, _p, _p, _p, _i, _i, _i, _i, _f, _i, _i])
_decl("molot_attn_decode_gqa", [_p, _p, _p, _p, _i, _i, _i, _i, _f])
_decl("molot_attn_decode_gqa_win", [_p, _p, _p, _p, _i, _i, _i, _i, _f, _i, _i])
_decl("molot_attn_decode_head_win", [_p, _p, _p, _p, _i, _i, _f, _i, _i])
_decl("molot_attn_decode_head", [_p, _p, _p, _p, _i, _i, _f])
_decl("molot_rope_apply", [_p, _i, _i, _p])
_decl("molot_rope_inv_freq", [_f, _i, _p])
_decl("molot_attn_decode_strided_dev", [_p, _p, _p, _p, _i, _i, _i, _i, _ll, _ll, _f, _i, _i, _p])
_decl("molot_norm_rope_append_dev",
      [_p, _p, _p, _p, _p, _p, _i, _f, _p, _i, _p, _p, _i, _i, _i, _i, _p])
_decl("molot_kv_create", [_i, _i, _i, _i, _pp])
_decl("molot_kv_create_ex", [_i, _i, _i, _i, _i, _pp])
_decl("molot_kv_dtype", [_p])
_decl("molot_kv_destroy", [_p], None)
_decl("molot_kv_length", [_p, _i])
_decl("molot_kv_set_length", [_p, _i, _i])
_decl("molot_kv_layer_data", [_p, _i, _pp, _pp])
_decl("molot_kv_write", [_p, _i, _i, _i, _p, _p, _p])
_decl("molot_attn_append_rope", [_p, _i, _p, _p, _p, _p, _p, _p, _i, _f, _p, _i, _i, _p])
_decl("molot_attn_decode", [_p, _i, _p, _p, _i, _f, _i, _i, _p])
_decl("molot_kv_check", [_p, _p])
_decl("molot_attn_step", [_p, _i, _p, _p, _p, _p, _p, _i, _f, _p, _i, _p, _i, _f, _i, _p])
_decl("molot_attn_prefill_gqa", [_p, _p, _p, _p, _i, _i, _i, _i, _i, _f, _i, _i])
_decl("molot_attn_prefill_strided_dev",
      [_p, _p, _p, _p, _i, _i, _i, _i, _i, _ll, _ll, _f, _i, _i, _p])
_decl("molot_attn_append_rope_tokens",
      [_p, _i, _p, _p, _p, _p, _p, _p, _i, _f, _p, _i, _i, _i, _p])
_decl("molot_attn_prefill", [_p, _i, _p, _p, _i, _i, _f, _i, _i, _p])
_decl("molot_gemv_q4", [_p, _p, _p, _p, _i, _i, _p, _p])
_decl("molot_pager_create", [_i, _i, _i, _i, _i, _i, _i, _pp])
_decl("molot_pager_create_ex", [_i, _i, _i, _i, _i, _i, _i, _i, _pp])
_decl("molot_paged_plan_set_kv_dtype", [_p, _i])
_decl("molot_pager_destroy", [_p], None)
_decl("molot_pager_add", [_p, _i, _p])
_decl("molot_pager_grow", [_p, _i, _i])
_decl("molot_pager_free", [_p, _i])
_decl("molot_pager_length", [_p, _i])
_decl("molot_pager_free_pages", [_p])
_decl("molot_pager_tables", [_p, _p, _i, _p, _p])
_decl("molot_pager_layer_pools", [_p, _i, _pp, _pp])
_decl("molot_gemv_q4_dev", [_p, _p, _p, _i, _i, _p, _p, _p])
_decl("molot_paged_plan_create", [_pp])
_decl("molot_paged_plan_destroy", [_p], None)
_decl("molot_paged_plan_build", [_p, _i, _i, _i, _i, _p, _p, _i, _p])
_decl("molot_paged_decode", [_p, _p, _p, _p, _p, _p, _i, _i, _f, _p])
_decl("molot_paged_append", [_p, _p, _p, _p, _p, _p, _p, _i, _f, _p, _p, _p, _p, _i, _i, _p])
_decl("molot_paged_check", [_p, _p])
_decl("molot_debug_withhold_next", [ctypes.c_ulonglong])
_decl("molot_noalloc_status", [_p, _i])
_decl("molot_comm_create", [_i, _i, ctypes.c_size_t, _pp])
_decl("molot_comm_handle", [_p, _p])
_decl("molot_comm_open", [_p, _p])
_decl("molot_comm_buffer", [_p, _pp])
_decl("molot_comm_wait", [_p, _p])
_decl("molot_comm_check", [_p, _p])
_decl("molot_comm_destroy", [_p], None)
_decl("molot_paged_decode_gather",
      [_p, _p, _p, ctypes.c_size_t, _p, _p, _p, _i, _i, _f, _p])

COMM_HANDLE_BYTES = 64
COMM_MAX_RANKS = 8


def library():
    """The loaded ctypes library (for callers binding extra symbols)."""
    return _lib


def header_symbols(path: str = HEADER) -> list[str]:
    """Every function the public header declares."""
    text = open(path).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(molot_[a-z0-9_]+)\s*\(", text)))


def status_string(status: int) -> str:
    return _lib.molot_status_string(status).decode()


def last_error() -> str:
    return _lib.molot_last_error().decode()


def check(status: int) -> None:
    if status != OK:
        raise MolotError(status, status_string(status), last_error())


# ------------------------------------------------------------------ helpers

def _host_f32(a) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.float32)
    return a


def _ptr(a) -> int | None:
    if a is None:
        return None
    if isinstance(a, np.ndarray):
        return a.ctypes.data
    if hasattr(a, "data_ptr"):  # torch tensor
        if not a.is_contiguous():
            raise ValueError("tensor must be contiguous")
        return a.data_ptr()
    return int(a)


def _stream_ptr(stream) -> int | None:
    if stream is None:
        try:
            import torch
            return torch.cuda.current_stream().cuda_stream
        except Exception:  # pragma: no cover - torch absent
            return None
    if hasattr(stream, "cuda_stream"):
        return stream.cuda_stream
    return int(stream)


def _check_cuda_tensor(t, name):
    if not (hasattr(t, "is_cuda") and t.is_cuda):
        raise ValueError(f"{name} must be a CUDA tensor")
    if t.dtype.__repr__() != "torch.float32" and str(t.dtype) != "torch.float32":
        raise ValueError(f"{name} must be float32")


class _CudaArray:
    """Minimal __cuda_array_interface__ exporter used to view library-owned
    device memory as a torch tensor without copying."""

    def __init__(self, ptr: int, shape: tuple, typestr: str = "<f4"):
        self.__cuda_array_interface__ = {
            "data": (ptr, False), "shape": tuple(shape), "typestr": typestr, "version": 3,
            "strides": None,
        }


# ------------------------------------------------------------------ host drop-ins

def attn_decode_gqa_cache(Q, K, V, nq, nkv, n, qhd, scale, pos_cur, window) -> np.ndarray:
    """attn.h:125-177 on host arrays: Q [nq*qhd], K/V [n][nkv*qhd] -> O [nq][qhd]."""
    Q, K, V = _host_f32(Q), _host_f32(K), _host_f32(V)
    O = np.zeros((nq, qhd), np.float32)
    check(_lib.molot_attn_decode_gqa_cache(_ptr(Q), _ptr(K), _ptr(V), _ptr(O), nq, nkv, n, qhd,
                                           scale, pos_cur, window))
    return O


def attn_prefill_gqa(Qm, K, V, nq, nkv, M, N, d, scale, pos0, window) -> np.ndarray:
    """gemm.h:409-446 on host arrays: Qm [M][nq][d], K/V [N][nkv*d] -> Om [M][nq][d]."""
    Qm, K, V = _host_f32(Qm), _host_f32(K), _host_f32(V)
    Om = np.zeros((M, nq, d), np.float32)
    check(_lib.molot_attn_prefill_gqa(_ptr(Qm), _ptr(K), _ptr(V), _ptr(Om), nq, nkv, M, N, d,
                                      scale, pos0, window))
    return Om


def prefill_strided(Q, K, V, O, nq, nkv, M, N, d, stride_t, stride_h, scale, pos0, window,
                    stream=None) -> None:
    """gemm.h:409-446 on device tensors: Q, O [M][nq][d]; slot t of kv head g
    at K + t*stride_t + g*stride_h."""
    check(_lib.molot_attn_prefill_strided_dev(_ptr(Q), _ptr(K), _ptr(V), _ptr(O), nq, nkv, M, N,
                                              d, stride_t, stride_h, scale, pos0, window,
                                              _stream_ptr(stream)))


def gemv_q4(q4, x) -> np.ndarray:
    """gemm.h:223-254 on host arrays: q4 = (scales f32 [rows][cols/32], zeros
    i8, data u8 [rows][cols/2], wsums i16) as quant.h lays a Q4Matrix out;
    returns y = W x [rows]."""
    sc, z, data, ws = (np.ascontiguousarray(a) for a in q4)
    rows, ng = sc.shape
    x = _host_f32(x)
    y = np.zeros(rows, np.float32)
    check(_lib.molot_gemv_q4(_ptr(sc), _ptr(z), _ptr(data), _ptr(ws), rows, ng * 32, _ptr(x),
                             _ptr(y)))
    return y


def gemv_q4_dev(scales, zeros, data, x, y, stream=None) -> None:
    """molot_gemv_q4_dev on device tensors (scales [rows][cols/32] f32, zeros
    int8, data uint8 [rows][cols/2], x [cols], y [rows])."""
    rows, ng = scales.shape
    check(_lib.molot_gemv_q4_dev(_ptr(scales), _ptr(zeros), _ptr(data), rows, ng * 32, _ptr(x),
                                 _ptr(y), _stream_ptr(stream)))


def attn_decode_gqa(Q, K, V, nq, nkv, n, d, scale) -> np.ndarray:
    """attn.h:111-120: K/V [nkv][n][d]."""
    Q, K, V = _host_f32(Q), _host_f32(K), _host_f32(V)
    O = np.zeros((nq, d), np.float32)
    check(_lib.molot_attn_decode_gqa(_ptr(Q), _ptr(K), _ptr(V), _ptr(O), nq, nkv, n, d, scale))
    return O


def attn_decode_gqa_win(Q, K, V, nq, nkv, n, d, scale, pos_cur, window) -> np.ndarray:
    """attn.h:178-187: K/V [nkv][n][d], sliding window."""
    Q, K, V = _host_f32(Q), _host_f32(K), _host_f32(V)
    O = np.zeros((nq, d), np.float32)
    check(_lib.molot_attn_decode_gqa_win(_ptr(Q), _ptr(K), _ptr(V), _ptr(O), nq, nkv, n, d, scale,
                                         pos_cur, window))
    return O


def attn_decode_head_win(Q, K, V, n, d, scale, pos_cur, window) -> np.ndarray:
    """attn.h:57-101: one head, K/V [n][d]."""
    Q, K, V = _host_f32(Q), _host_f32(K), _host_f32(V)
    out = np.zeros(d, np.float32)
    check(_lib.molot_attn_decode_head_win(_ptr(Q), _ptr(K), _ptr(V), _ptr(out), n, d, scale,
                                          pos_cur, window))
    return out


def attn_decode_head(Q, K, V, n, d, scale) -> np.ndarray:
    """attn.h:104-107."""
    Q, K, V = _host_f32(Q), _host_f32(K), _host_f32(V)
    out = np.zeros(d, np.float32)
    check(_lib.molot_attn_decode_head(_ptr(Q), _ptr(K), _ptr(V), _ptr(out), n, d, scale))
    return out


def rope_apply(x, d, pos, inv_freq) -> np.ndarray:
    """attn.h:19-28 on one head vector (returns the rotated copy)."""
    x = _host_f32(x).copy()
    f = _host_f32(inv_freq)
    check(_lib.molot_rope_apply(_ptr(x), d, pos, _ptr(f)))
    return x


def rope_inv_freq(base, d) -> np.ndarray:
    """attn.h:31-33."""
    out = np.zeros(d // 2, np.float32)
    check(_lib.molot_rope_inv_freq(base, d, _ptr(out)))
    return out


def device_status(clear: bool = True) -> int:
    """Device-side status of the current device's default workspace and of
    its no-alloc scratch (0 or ERR_TIMEOUT)."""
    return _lib.molot_device_status(1 if clear else 0)


def noalloc_status(stream=None, clear: bool = True) -> int:
    """Status word of the no-alloc scratch (molot_noalloc_status): 0, or
    ERR_TIMEOUT when a no-alloc decode gave up on a bounded wait."""
    return _lib.molot_noalloc_status(_stream_ptr(stream), 1 if clear else 0)


def debug_withhold_next(wait_limit_ns: int) -> None:
    """Failure-detection test hook (molot_debug_withhold_next): the calling
    thread's next decode launch withholds its copies so its first bounded
    wait runs out after wait_limit_ns; 0 cancels."""
    check(_lib.molot_debug_withhold_next(int(wait_limit_ns)))


# ------------------------------------------------------------------ device forms

def decode_strided(Q, K, V, O, nq, nkv, n, d, stride_t, stride_h, scale, pos_cur, window,
                   stream=None) -> None:
    """Stream-ordered decode over a strided contiguous cache (torch tensors)."""
    check(_lib.molot_attn_decode_strided_dev(_ptr(Q), _ptr(K), _ptr(V), _ptr(O), nq, nkv, n, d,
                                             stride_t, stride_h, scale, pos_cur, window,
                                             _stream_ptr(stream)))


def norm_rope_append(q, k, v, q_out, q_norm, k_norm, v_norm, eps, freq, pos, kc, vc, slot, nq,
                     nkv, d, stream=None) -> None:
    """forward.h:554-575 on device tensors for a [cap][nkv*d] cache."""
    check(_lib.molot_norm_rope_append_dev(_ptr(q), _ptr(k), _ptr(v), _ptr(q_out), _ptr(q_norm),
                                          _ptr(k_norm), int(v_norm), eps, _ptr(freq), pos,
                                          _ptr(kc), _ptr(vc), slot, nq, nkv, d,
                                          _stream_ptr(stream)))


class KVCache:
    """HBM-resident per-layer KV cache (replaces forward.h's Runner::KVC)."""

    def __init__(self, n_layers: int, nkv: int, hd: int, cap: int, dtype: str = "f32"):
        if dtype not in _KV_DTYPES:
            raise ValueError("dtype must be 'f32', 'bf16' or 'q8'")
        h = ctypes.c_void_p()
        check(_lib.molot_kv_create_ex(n_layers, nkv, hd, cap, _KV_DTYPES[dtype],
                                      ctypes.byref(h)))
        self._h = h
        self.n_layers, self.nkv, self.hd, self.cap = n_layers, nkv, hd, cap
        self.dtype = dtype

    def close(self) -> None:
        if getattr(self, "_h", None):
            _lib.molot_kv_destroy(self._h)
            self._h = None

    def __del__(self):  # pragma: no cover - best effort
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self):
        return self._h

    def length(self, layer: int) -> int:
        r = _lib.molot_kv_length(self._h, layer)
        if r < 0:
            check(r)
        return r

    def set_length(self, layer: int, n: int) -> None:
        check(_lib.molot_kv_set_length(self._h, layer, n))

    def layer_ptrs(self, layer: int) -> tuple[int, int]:
        k = ctypes.c_void_p()
        v = ctypes.c_void_p()
        check(_lib.molot_kv_layer_data(self._h, layer, ctypes.byref(k), ctypes.byref(v)))
        return k.value, v.value

    def layer_tensors(self, layer: int):
        """(K, V) torch views [nkv][cap][hd] (head-major) of the layer's
        device memory: float32, or bfloat16 for a bf16 cache; a q8 cache
        gives uint8 [nkv][cap][q8_row_bytes(hd)] (see q8_unpack)."""
        import torch
        kp, vp = self.layer_ptrs(layer)
        shape = (self.nkv, self.cap, self.hd)
        if self.dtype == "q8":
            shape = (self.nkv, self.cap, q8_row_bytes(self.hd))
            return (torch.as_tensor(_CudaArray(kp, shape, "|u1"), device="cuda"),
                    torch.as_tensor(_CudaArray(vp, shape, "|u1"), device="cuda"))
        if self.dtype == "bf16":
            return (torch.as_tensor(_CudaArray(kp, shape, "<i2"), device="cuda").view(torch.bfloat16),
                    torch.as_tensor(_CudaArray(vp, shape, "<i2"), device="cuda").view(torch.bfloat16))
        return (torch.as_tensor(_CudaArray(kp, shape), device="cuda"),
                torch.as_tensor(_CudaArray(vp, shape), device="cuda"))

    def write(self, layer: int, slot0: int, k, v, stream=None) -> None:
        rows = k.shape[0]
        check(_lib.molot_kv_write(self._h, layer, slot0, rows, _ptr(k), _ptr(v),
                                  _stream_ptr(stream)))

    def append_rope(self, layer, q, k, v, q_out, q_norm=None, k_norm=None, v_norm=False,
                    eps=1e-6, freq=None, pos=0, nq=None, stream=None) -> None:
        nq = nq if nq is not None else q.numel() // self.hd
        check(_lib.molot_attn_append_rope(self._h, layer, _ptr(q), _ptr(k), _ptr(v), _ptr(q_out),
                                          _ptr(q_norm), _ptr(k_norm), int(v_norm), eps,
                                          _ptr(freq), pos, nq, _stream_ptr(stream)))

    def step(self, layer, q, k, v, o, scale, pos, window=0, q_norm=None, k_norm=None,
             v_norm=False, eps=1e-6, freq=None, nq=None, stream=None) -> None:
        """forward.h:554-590 in one launch: prologue on the raw q/k/v, append
        at slot n, attention into o."""
        nq = nq if nq is not None else q.numel() // self.hd
        check(_lib.molot_attn_step(self._h, layer, _ptr(q), _ptr(k), _ptr(v), _ptr(q_norm),
                                   _ptr(k_norm), int(v_norm), eps, _ptr(freq), pos, _ptr(o), nq,
                                   scale, window, _stream_ptr(stream)))

    def append_rope_tokens(self, layer, q, k, v, q_out, q_norm=None, k_norm=None, v_norm=False,
                           eps=1e-6, freq=None, pos0=0, M=None, nq=None, stream=None) -> None:
        """forward.h:368-392: M tokens' prologue, rows appended at n..n+M-1."""
        M = M if M is not None else k.numel() // (self.nkv * self.hd)
        nq = nq if nq is not None else q.numel() // (M * self.hd)
        check(_lib.molot_attn_append_rope_tokens(self._h, layer, _ptr(q), _ptr(k), _ptr(v),
                                                 _ptr(q_out), _ptr(q_norm), _ptr(k_norm),
                                                 int(v_norm), eps, _ptr(freq), pos0, M, nq,
                                                 _stream_ptr(stream)))

    def prefill(self, src_layer, q, o, scale, pos0, window=0, M=None, nq=None,
                stream=None) -> None:
        """gemm.h:409-446 over src_layer's cache: q, o [M][nq][hd]."""
        if M is None or nq is None:
            if q.dim() == 3:
                M, nq = q.shape[0], q.shape[1]
            else:
                raise ValueError("pass M and nq for flat q")
        check(_lib.molot_attn_prefill(self._h, src_layer, _ptr(q), _ptr(o), nq, M, scale, pos0,
                                      window, _stream_ptr(stream)))

    def decode(self, src_layer, q, o, scale, pos_cur, window=0, nq=None, stream=None) -> None:
        nq = nq if nq is not None else q.numel() // self.hd
        check(_lib.molot_attn_decode(self._h, src_layer, _ptr(q), _ptr(o), nq, scale, pos_cur,
                                     window, _stream_ptr(stream)))

    def check(self, stream=None) -> None:
        check(_lib.molot_kv_check(self._h, _stream_ptr(stream)))


class Pager:
    """Continuous-batching page manager (molot_pager_*): sequences, their
    pages and lengths, block tables for a batch, optional HBM page pools."""

    def __init__(self, n_layers, nkv, d, page_size, num_pages, max_seqs, max_pages_per_seq,
                 dtype: str = "f32"):
        if dtype not in _KV_DTYPES:
            raise ValueError("dtype must be 'f32', 'bf16' or 'q8'")
        h = ctypes.c_void_p()
        check(_lib.molot_pager_create_ex(n_layers, nkv, d, page_size, num_pages, max_seqs,
                                         max_pages_per_seq, _KV_DTYPES[dtype], ctypes.byref(h)))
        self._h = h
        self.dtype = dtype
        self.n_layers, self.nkv, self.d, self.page_size = n_layers, nkv, d, page_size
        self.num_pages, self.max_pages = num_pages, max_pages_per_seq

    def close(self) -> None:
        if getattr(self, "_h", None):
            _lib.molot_pager_destroy(self._h)
            self._h = None

    def __del__(self):  # pragma: no cover
        try:
            self.close()
        except Exception:
            pass

    def add(self, slots: int) -> int:
        s = ctypes.c_int()
        check(_lib.molot_pager_add(self._h, slots, ctypes.byref(s)))
        return s.value

    def grow(self, seq: int, n_new: int = 1) -> None:
        check(_lib.molot_pager_grow(self._h, seq, n_new))

    def free(self, seq: int) -> None:
        check(_lib.molot_pager_free(self._h, seq))

    def length(self, seq: int) -> int:
        r = _lib.molot_pager_length(self._h, seq)
        if r < 0:
            check(r)
        return r

    def free_pages(self) -> int:
        return _lib.molot_pager_free_pages(self._h)

    def tables(self, seqs):
        """(block_table int32 [B][max_pages], seq_lens int32 [B]) on the host."""
        sq = np.ascontiguousarray(seqs, dtype=np.int32)
        bt = np.zeros((sq.size, self.max_pages), np.int32)
        lens = np.zeros(sq.size, np.int32)
        check(_lib.molot_pager_tables(self._h, _ptr(sq), sq.size, _ptr(bt), _ptr(lens)))
        return bt, lens

    def layer_pools(self, layer: int):
        """(K, V) torch views [num_pages][nkv][page_size][d] of a layer's pools:
        float32, bfloat16 for bf16 pools, uint8 rows of q8_row_bytes(d) for
        q8 pools."""
        import torch
        k = ctypes.c_void_p()
        v = ctypes.c_void_p()
        check(_lib.molot_pager_layer_pools(self._h, layer, ctypes.byref(k), ctypes.byref(v)))
        shape = (self.num_pages, self.nkv, self.page_size, self.d)
        if self.dtype == "q8":
            shape = shape[:3] + (q8_row_bytes(self.d),)
            return (torch.as_tensor(_CudaArray(k.value, shape, "|u1"), device="cuda"),
                    torch.as_tensor(_CudaArray(v.value, shape, "|u1"), device="cuda"))
        if self.dtype == "bf16":
            return (torch.as_tensor(_CudaArray(k.value, shape, "<i2"),
                                    device="cuda").view(torch.bfloat16),
                    torch.as_tensor(_CudaArray(v.value, shape, "<i2"),
                                    device="cuda").view(torch.bfloat16))
        return (torch.as_tensor(_CudaArray(k.value, shape), device="cuda"),
                torch.as_tensor(_CudaArray(v.value, shape), device="cuda"))


class PagedPlan:
    """Batch shape of one decode step over a paged pool (see molot_b200.h)."""

    def __init__(self, dtype: str = "f32"):
        """dtype: element type of the pools it is used with ('f32', 'bf16', 'q8')."""
        if dtype not in _KV_DTYPES:
            raise ValueError("dtype must be 'f32', 'bf16' or 'q8'")
        h = ctypes.c_void_p()
        check(_lib.molot_paged_plan_create(ctypes.byref(h)))
        self._h = h
        check(_lib.molot_paged_plan_set_kv_dtype(h, _KV_DTYPES[dtype]))

    def close(self) -> None:
        if getattr(self, "_h", None):
            _lib.molot_paged_plan_destroy(self._h)
            self._h = None

    def __del__(self):  # pragma: no cover
        try:
            self.close()
        except Exception:
            pass

    def build(self, nq, nkv, d, seq_lens, positions=None, window=0, stream=None) -> None:
        sl = np.ascontiguousarray(seq_lens, dtype=np.int32)
        pos = None if positions is None else np.ascontiguousarray(positions, dtype=np.int32)
        self._keep = (sl, pos)
        check(_lib.molot_paged_plan_build(self._h, sl.size, nq, nkv, d, _ptr(sl), _ptr(pos),
                                          window, _stream_ptr(stream)))

    def decode(self, Q, O, k_pool, v_pool, block_table, page_size, scale, stream=None) -> None:
        check(_lib.molot_paged_decode(self._h, _ptr(Q), _ptr(O), _ptr(k_pool), _ptr(v_pool),
                                      _ptr(block_table), block_table.shape[1], page_size, scale,
                                      _stream_ptr(stream)))

    def append(self, q, k, v, q_out, k_pool, v_pool, block_table, page_size, q_norm=None,
               k_norm=None, v_norm=False, eps=1e-6, freq=None, stream=None) -> None:
        check(_lib.molot_paged_append(self._h, _ptr(q), _ptr(k), _ptr(v), _ptr(q_out),
                                      _ptr(q_norm), _ptr(k_norm), int(v_norm), eps, _ptr(freq),
                                      _ptr(k_pool), _ptr(v_pool), _ptr(block_table),
                                      block_table.shape[1], page_size, _stream_ptr(stream)))

    def decode_gather(self, comm, Q, out_offset, k_pool, v_pool, block_table, page_size, scale,
                      stream=None) -> None:
        """molot_paged_decode_gather: outputs into every rank's gathered
        buffer of `comm` at float offset out_offset ([B][nranks*nq][d])."""
        check(_lib.molot_paged_decode_gather(self._h, comm.handle, _ptr(Q), int(out_offset),
                                             _ptr(k_pool), _ptr(v_pool), _ptr(block_table),
                                             block_table.shape[1], page_size, scale,
                                             _stream_ptr(stream)))

    def check(self, stream=None) -> None:
        check(_lib.molot_paged_check(self._h, _stream_ptr(stream)))


class Comm:
    """Peer-gather group for kv-head sharding (molot_comm_*): one process per
    GPU; every rank's gathering decode writes its heads' outputs straight
    into every rank's buffer over NVLink.  The caller exchanges the 64-byte
    handles (`handle()`) between ranks and passes all of them to `open()`."""

    def __init__(self, nranks: int, rank: int, buf_bytes: int):
        h = ctypes.c_void_p()
        check(_lib.molot_comm_create(nranks, rank, buf_bytes, ctypes.byref(h)))
        self._h = h
        self.nranks, self.rank, self.buf_bytes = nranks, rank, buf_bytes

    @property
    def handle(self):
        return self._h

    def ipc_handle(self) -> bytes:
        buf = ctypes.create_string_buffer(COMM_HANDLE_BYTES)
        check(_lib.molot_comm_handle(self._h, buf))
        return buf.raw

    def open(self, handles) -> None:
        """handles: the nranks byte strings of ipc_handle(), in rank order."""
        if len(handles) != self.nranks:
            raise ValueError("one handle per rank")
        blob = b"".join(bytes(x) for x in handles)
        if len(blob) != COMM_HANDLE_BYTES * self.nranks:
            raise ValueError("bad handle size")
        buf = ctypes.create_string_buffer(blob, len(blob))
        check(_lib.molot_comm_open(self._h, buf))

    def buffer(self, shape, offset: int = 0):
        """torch float32 view of the gathered buffer from float `offset`."""
        import torch
        p = ctypes.c_void_p()
        check(_lib.molot_comm_buffer(self._h, ctypes.byref(p)))
        n = 1
        for x in shape:
            n *= int(x)
        if (offset + n) * 4 > self.buf_bytes:
            raise ValueError("view outside the comm buffer")
        return torch.as_tensor(_CudaArray(p.value + 4 * offset, tuple(shape)), device="cuda")

    def wait(self, stream=None) -> None:
        check(_lib.molot_comm_wait(self._h, _stream_ptr(stream)))

    def check(self, stream=None) -> None:
        check(_lib.molot_comm_check(self._h, _stream_ptr(stream)))

    def close(self) -> None:
        if getattr(self, "_h", None):
            _lib.molot_comm_destroy(self._h)
            self._h = None

    def __del__(self):  # pragma: no cover
        try:
            self.close()
        except Exception:
            pass
