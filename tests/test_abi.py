"""The C-ABI library builds, loads, and exports every symbol include/bebelm_attn.h declares (CPU only)."""
import ctypes as C
import os
import re

import pytest

import bebelm_b200 as bb

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    hdr = open(os.path.join(ROOT, "include", "bebelm_attn.h")).read()
    return sorted(set(re.findall(r"^BEBELM_API\s+int\s+(bebelm_\w+)\s*\(", hdr, flags=re.M)))


def test_header_matches_python_binding():
    assert declared_symbols() == sorted(bb.EXPORTS)


def test_library_exports_every_declared_symbol():
    L = bb.load_library()
    for name in declared_symbols():
        assert hasattr(L, name), name
    assert L.bebelm_abi_version() == 1


def test_no_device_fails_loudly():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is visible")
    L = bb.load_library()
    n = C.c_int(-1)
    assert L.bebelm_device_count(C.byref(n)) == 0 and n.value == 0
    h = C.c_void_p()
    rc = L.bebelm_kv_create(6, 8, 64, 1024, 64, 0, 0, C.byref(h))
    assert rc == bb.ERR_NO_DEVICE
    assert "device" in bb.last_error()
    with pytest.raises(bb.BebelmError):
        bb.attention_decode([1.0, 0.0], [1.0, 0.0], [5.0, 7.0], 1, 1, 1, 2)


def test_argument_validation_without_device():
    L = bb.load_library()
    assert L.bebelm_kv_create(6, 8, 32, 1024, 64, 0, 0, C.byref(C.c_void_p())) == bb.ERR_UNSUPPORTED
    assert L.bebelm_kv_create(6, 8, 64, 1024, 32, 0, 0, C.byref(C.c_void_p())) == bb.ERR_UNSUPPORTED
    assert L.bebelm_kv_create(6, 8, 64, 1024, 64, 7, 0, C.byref(C.c_void_p())) == bb.ERR_UNSUPPORTED  # unknown dtype
    assert L.bebelm_kv_len(None, C.byref(C.c_size_t())) == bb.ERR_INVALID
    assert L.bebelm_attn_decode_host(None, None, None, 1, 3, 2, 64, None) == bb.ERR_INVALID
    buf = C.create_string_buffer(64)
    assert L.bebelm_last_error(buf, 64) == 0 and buf.value

    # logits head and greedy sampling: argument errors come before any device work
    assert L.bebelm_head_create(0, 12, None, 2048, 100, None, C.byref(C.c_void_p())) == bb.ERR_INVALID
    assert L.bebelm_head_logits(None, None, 1e-5, None, None, 0, None) == bb.ERR_INVALID
    assert L.bebelm_sample_greedy(None, 4, None, 0, 1.0, None, 0, None) == bb.ERR_INVALID
    lg = (C.c_float * 2)(1.0, 2.0)
    hist = (C.c_uint32 * 1)(5)
    tok = C.c_uint32()
    assert L.bebelm_sample_greedy(lg, 2, hist, 1, 2.0, C.byref(tok), 0, None) == bb.ERR_INVALID  # id >= n
