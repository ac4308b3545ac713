"""The C-ABI library: it loads, exports every symbol the public header
declares, and rejects bad arguments before touching a device (no GPU here)."""
import ctypes
import os
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def lib():
    import molot_b200
    return molot_b200


def test_library_loads_and_exports_header(lib):
    syms = lib.header_symbols()
    assert "molot_attn_decode_gqa_cache" in syms and "molot_paged_decode" in syms
    out = subprocess.run(["nm", "-D", "--defined-only", lib.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = [s for s in syms if s not in exported]
    assert not missing, missing
    for s in syms:
        getattr(lib.library(), s)


def test_status_strings(lib):
    assert lib.status_string(0) == "ok"
    assert lib.status_string(lib.ERR_CACHE_FULL) == "KV cache full"
    assert lib.status_string(lib.ERR_CACHE_EMPTY) == "shared KV empty"
    assert lib.status_string(12345) == "unknown status"


def test_bad_shapes_rejected_without_device(lib):
    L = lib.library()
    # nq not a multiple of nkv
    rc = L.molot_attn_decode_strided_dev(None, None, None, None, 3, 2, 10, 128, 256, 128, 1.0, 9,
                                         0, None)
    assert rc == lib.ERR_INVALID
    # head dim without a kernel
    rc = L.molot_attn_decode_strided_dev(None, None, None, None, 4, 2, 10, 72, 144, 72, 1.0, 9, 0,
                                         None)
    assert rc == lib.ERR_UNSUPPORTED
    assert "head_dim" in lib.last_error()
    # host drop-in with null buffers
    assert L.molot_attn_decode_gqa_cache(None, None, None, None, 4, 2, 10, 128, 1.0, 9, 0) == \
        lib.ERR_INVALID
    # kv handle with zero sizes
    h = ctypes.c_void_p()
    assert L.molot_kv_create(0, 8, 128, 16, ctypes.byref(h)) == lib.ERR_INVALID
    assert L.molot_rope_inv_freq(1e4, 0, None) == lib.ERR_INVALID


def test_rope_inv_freq_host_table(lib):
    import oracle
    got = lib.rope_inv_freq(5e5, 128)
    want = oracle.rope_inv_freq(5e5, 128)
    assert np.max(np.abs(got - want) / want) < 1e-6


def test_python_errors_carry_status(lib):
    with pytest.raises(lib.MolotError) as ei:
        lib.check(lib.ERR_INVALID)
    assert ei.value.status == lib.ERR_INVALID


def test_product_does_not_reference_oracle():
    """The shipped library and package never load the checker."""
    for root, _, files in os.walk(os.path.join(ROOT, "molot_b200")):
        for f in files:
            if f.endswith((".py", ".cu", ".cuh", ".h")):
                text = open(os.path.join(root, f)).read()
                assert "import oracle" not in text and "attn_oracle" not in text, f
    out = subprocess.run(["nm", "-D", os.path.join(ROOT, "molot_b200", "libmolot_b200.so")],
                         capture_output=True, text=True, check=True).stdout
    assert "oracle_" not in out and "ref_attn" not in out


def test_comm_and_hooks_validate_without_device(lib):
    """The peer-gather group and the test hook reject bad arguments before
    any CUDA call."""
    L = lib.library()
    h = ctypes.c_void_p()
    assert L.molot_comm_create(0, 0, 1024, ctypes.byref(h)) == lib.ERR_INVALID
    assert L.molot_comm_create(9, 0, 1024, ctypes.byref(h)) == lib.ERR_INVALID
    assert L.molot_comm_create(2, 2, 1024, ctypes.byref(h)) == lib.ERR_INVALID
    assert L.molot_comm_create(2, -1, 1024, ctypes.byref(h)) == lib.ERR_INVALID
    assert L.molot_comm_create(2, 0, 1000, ctypes.byref(h)) == lib.ERR_INVALID  # not 16-aligned
    assert L.molot_comm_create(2, 0, 0, ctypes.byref(h)) == lib.ERR_INVALID
    assert L.molot_comm_create(2, 0, 1024, None) == lib.ERR_INVALID
    assert L.molot_comm_handle(None, None) == lib.ERR_INVALID
    assert L.molot_comm_open(None, None) == lib.ERR_INVALID
    assert L.molot_comm_buffer(None, None) == lib.ERR_INVALID
    assert L.molot_comm_wait(None, None) == lib.ERR_INVALID
    assert L.molot_comm_check(None, None) == lib.ERR_INVALID
    L.molot_comm_destroy(None)
    assert L.molot_paged_decode_gather(None, None, None, 0, None, None, None, 1, 16, 1.0,
                                       None) == lib.ERR_INVALID
    # the hook only records a request; 0 cancels it
    assert L.molot_debug_withhold_next(1000) == lib.OK
    assert L.molot_debug_withhold_next(0) == lib.OK
    assert lib.COMM_HANDLE_BYTES == 64 and lib.COMM_MAX_RANKS == 8
