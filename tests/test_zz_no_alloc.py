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
        # the call left no timeout behind, and the pool's check (which also covers this
        # path's waits) reports a clean run
        assert L.bebelm_kv_check(cache._h, stream) == 0, bb.last_error()
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
    assert "split counters" in bb.last_error() and "no-allocation" in bb.last_error()
    cache.close()


def test_noalloc_rejects_window_beyond_partial_region():
    torch = pytest.importorskip("torch")
    L = bb.load_library()
    # 1024 kv heads (one split counter each, within the limit) over a 500-page window: the split
    # plan caps a split at 256 pages, so 2 splits x 1024 heads x 4 query heads x 66 floats of
    # partial results, more than the array's partial region. bf16 pages keep the pool at ~8.4 GB.
    n_kv, n_pos = 1024, 500 * 64
    cache = bb.Cache(n_layers=1, n_kv_heads=n_kv, max_context=n_pos, kv_dtype=bb.BF16)
    rows = torch.zeros((2048, n_kv * D), device="cuda")
    for _ in range(n_pos // 2048):
        cache.append(0, rows, rows)
    cache.append(0, rows[: n_pos % 2048], rows[: n_pos % 2048])
    assert cache.layer_len(0) == n_pos
    del rows
    q = torch.zeros(4 * n_kv * D, device="cuda")
    out = torch.zeros(4 * n_kv * D, device="cuda")
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = L.bebelm_attn_decode_cached_noalloc(cache._h, 0, 4 * n_kv, C.c_void_p(q.data_ptr()),
                                             C.c_void_p(out.data_ptr()), stream)
    assert rc == bb.ERR_INVALID
    msg = bb.last_error()
    assert "scratch floats" in msg and "no-allocation" in msg, msg
    # the regular entry point serves the same window (it grows its scratch)
    rc = L.bebelm_attn_decode_cached(cache._h, 0, 4 * n_kv, C.c_void_p(q.data_ptr()), C.c_void_p(out.data_ptr()),
                                     bb.MEM_DEVICE, stream)
    assert rc == 0, bb.last_error()
    assert L.bebelm_kv_check(cache._h, stream) == 0
    cache.close()
    torch.cuda.empty_cache()


def test_expired_wait_is_reported_and_the_next_call_is_correct():
    """A bounded device-side wait that gives up (forced through bebelm_debug_expire_next_wait:
    the first CTA waits, with a short limit, on a barrier nothing completes; no GPU fault) is
    reported, on the no-allocation path by bebelm_kv_check and on a host-memory call by the
    call itself, and leaves nothing behind: the split counters are cleared and the next call
    returns the same output as before the failure."""
    torch = pytest.importorskip("torch")
    L = bb.load_library()
    n = 16384  # 7 pages a split: more than the 3-stage ring, so the timed-out CTA has copies to wait for
    cache = bb.Cache(n_layers=1, max_context=n)
    for c0 in range(0, n, 4096):
        cache.append(0, oracle.normal(10 + c0, (4096, KVH * D)), oracle.normal(11 + c0, (4096, KVH * D)))
    qh = oracle.normal(12, (H * D,))
    q = torch.from_numpy(qh).cuda()
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    outs = [torch.full((H * D,), float("nan"), device="cuda") for _ in range(3)]

    def noalloc(o):
        return L.bebelm_attn_decode_cached_noalloc(cache._h, 0, H, C.c_void_p(q.data_ptr()),
                                                   C.c_void_p(o.data_ptr()), stream)

    assert noalloc(outs[0]) == 0, bb.last_error()
    assert L.bebelm_kv_check(cache._h, stream) == 0, bb.last_error()
    assert L.bebelm_debug_expire_next_wait(1) == 0
    assert noalloc(outs[1]) == 0, bb.last_error()  # device memory: the call only enqueues
    assert L.bebelm_kv_check(cache._h, stream) == bb.ERR_TIMEOUT
    assert "timed out" in bb.last_error()
    assert noalloc(outs[2]) == 0, bb.last_error()
    assert L.bebelm_kv_check(cache._h, stream) == 0, bb.last_error()
    assert torch.equal(outs[2], outs[0])

    # a host-memory call reports the timeout itself, and the next one is correct
    oh = np.full(H * D, np.nan, np.float32)
    assert L.bebelm_debug_expire_next_wait(1) == 0
    rc = L.bebelm_attn_decode_cached(cache._h, 0, H, C.c_void_p(qh.ctypes.data), C.c_void_p(oh.ctypes.data),
                                     bb.MEM_HOST, None)
    assert rc == bb.ERR_TIMEOUT, bb.last_error()
    rc = L.bebelm_attn_decode_cached(cache._h, 0, H, C.c_void_p(qh.ctypes.data), C.c_void_p(oh.ctypes.data),
                                     bb.MEM_HOST, None)
    assert rc == 0, bb.last_error()
    assert np.abs(oh - outs[0].cpu().numpy()).max() <= 1e-6  # the same split plan as the no-allocation path
    kw, vw = cache.read(0)
    ref = oracle.attention_decode(qh, kw, vw, kw.shape[0], H, KVH, D)
    assert np.abs(oh - ref).max() <= DECODE_ATOL
    assert L.bebelm_debug_expire_next_wait(0) == 0
    cache.close()
