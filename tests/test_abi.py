"""CPU tests of the C ABI boundary: the library loads, exports every function
include/laguna_cuda.h declares, and its host-only helpers behave (no GPU)."""
import ctypes as C
import os
import re

import numpy as np

from laguna_raw_halo_strix_b200 import lc

HEADER = os.path.join(os.path.dirname(__file__), "..", "include", "laguna_cuda.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    names = re.findall(r"^\s*(?:const\s+)?(?:int|void|uint64_t|uint32_t|float|size_t|const char)\s*\*?\s*(lc_\w+)\s*\(",
                       src, flags=re.M)
    return sorted(set(names))


def test_header_symbols_exported():
    L = lc.lib()
    names = declared_functions()
    assert len(names) >= 35, names
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing


def test_binding_covers_header():
    assert set(declared_functions()) <= set(lc.SIGNATURES), set(declared_functions()) - set(lc.SIGNATURES)


def test_version_and_errors():
    L = lc.lib()
    assert b"sm_100a" in L.lc_version()
    # null out-pointer is rejected with a message, nothing aborts
    assert L.lc_init(0, None) == lc.LC_ERR_INVALID
    assert "null" in lc.last_error()
    assert L.lc_set_half_mode(None, 0) == lc.LC_ERR_INVALID
    assert L.lc_buf_upload(None, None, 0) == lc.LC_ERR_INVALID


def test_keys_order_and_roundtrip():
    vals = np.array([-np.inf, -3.5, -1e-30, -0.0, 0.0, 1e-30, 2.0, 7.25, np.inf], np.float32)
    keys = [lc.pack_key(float(v), 5) for v in vals]
    s = [int(np.uint64(k).view(np.int64)) for k in keys]
    assert s == sorted(s) and len(set(s)) == len(s)
    # ties: larger index wins (src/lib.rs:456-464 keeps the last maximum)
    i64 = lambda k: int(np.uint64(k).view(np.int64))  # noqa: E731
    assert i64(lc.pack_key(1.0, 9)) > i64(lc.pack_key(1.0, 3))
    for v in vals:
        k = lc.pack_key(float(v), 123)
        assert lc.key_index(k) == 123
        got = lc.key_value(k)
        assert got == v and np.signbit(got) == np.signbit(v)


def test_rope_freq_matches_oracle(oracle):
    for dim, base in ((128, 500000.0), (64, 10000.0)):
        assert np.array_equal(lc.rope_freq(dim, base), oracle.rope_freq(dim, base))


def test_no_device_reports_error():
    import torch

    if torch.cuda.is_available():
        return
    h = C.c_void_p()
    st = lc.lib().lc_init(0, C.byref(h))
    assert st != lc.LC_OK and lc.last_error()
