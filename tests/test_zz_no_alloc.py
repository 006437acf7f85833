"""The no-allocation decode entry point matches the regular cached decode.

bebelm_attn_decode_cached_noalloc serves callers that cannot call cudaMalloc while
decoding; it keeps its split scratch in a fixed device array of the library instead of
growing pool scratch. This file is named to be collected last, so that a failure here
cannot hide any other test when the run stops at the first failure.
"""
import ctypes as C

import numpy as np
import pytest

import bebelm_b200 as bb
import oracle

pytestmark = pytest.mark.gpu

H, KVH, D = 32, 8, 64
DECODE_ATOL = 1e-3


def test_noalloc_decode_matches_cached_decode_twice():
    torch = pytest.importorskip("torch")
    L = bb.load_library()
    n = 5000
    cache = bb.Cache(n_layers=2, max_context=8192)
    k = oracle.normal(1, (n, KVH * D))
    v = oracle.normal(2, (n, KVH * D))
    cache.append(1, k, v)
    cache.evict_front(37)  # a window that does not start on a page boundary
    q = torch.from_numpy(oracle.normal(3, (H * D,))).cuda()
    want = torch.empty(H * D, device="cuda")
    got = torch.empty(H * D, device="cuda")
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = L.bebelm_attn_decode_cached(cache._h, 1, H, C.c_void_p(q.data_ptr()), C.c_void_p(want.data_ptr()),
                                     bb.MEM_DEVICE, stream)
    assert rc == 0, bb.last_error()
    for call in range(2):  # the second call reuses the array the first one left behind
        got.fill_(float("nan"))
        rc = L.bebelm_attn_decode_cached_noalloc(cache._h, 1, H, C.c_void_p(q.data_ptr()),
                                                 C.c_void_p(got.data_ptr()), stream)
        assert rc == 0, bb.last_error()
        torch.cuda.synchronize()
        err = (got - want).abs().max().item()
        assert err <= DECODE_ATOL, (call, err)
    # and both agree with the reference arithmetic
    kw, vw = cache.read(1)
    ref = oracle.attention_decode(q.cpu().numpy(), kw, vw, kw.shape[0], H, KVH, D)
    assert np.abs(got.cpu().numpy() - ref).max() <= DECODE_ATOL


def test_noalloc_rejects_oversized_window():
    torch = pytest.importorskip("torch")
    L = bb.load_library()
    # 8200 kv heads: one position already needs 8200 x 66 floats of split scratch,
    # more than the fixed array holds (the regular entry point would just allocate)
    n_kv = 8200
    cache = bb.Cache(n_layers=1, n_kv_heads=n_kv, max_context=64)
    row = torch.zeros((1, n_kv * D), device="cuda")
    cache.append(0, row, row)
    q = torch.zeros(n_kv * D, device="cuda")
    out = torch.zeros(n_kv * D, device="cuda")
    rc = L.bebelm_attn_decode_cached_noalloc(cache._h, 0, n_kv, C.c_void_p(q.data_ptr()), C.c_void_p(out.data_ptr()),
                                             C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == bb.ERR_INVALID
    assert "no-allocation" in bb.last_error()
    cache.close()
