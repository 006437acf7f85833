"""Pins the CPU oracle to the reference's own known-answer tests (CPU only)."""
import math

import numpy as np
import pytest

import oracle


def test_attention_kats(kats):
    for case in kats["attention"]:
        out = oracle.attention_decode(case["q"], case["k"], case["v"], case["n_ctx"], case["n_heads"],
                                      case["n_kv_heads"], case["head_dim"])
        want = np.array(case["out"], np.float32)
        if case.get("exact"):
            assert np.array_equal(out, want), case["src"]
        else:
            assert np.abs(out - want).max() < case["tol"], case["src"]


def test_softmax_kats(kats):
    for case in kats["softmax"]:
        out = oracle.softmax(case["x"])
        want = np.array(case["out"], np.float32)
        assert out.shape == want.shape
        if out.size:
            assert np.abs(out - want).max() < max(case["tol"], 1e-30), case["src"]
    out = oracle.softmax([1.0, 2.0, 3.0])
    assert abs(float(out.sum()) - 1.0) < 1e-6


def peaked_logits(c):
    i = np.arange(c["n"])
    return np.where(i < c["n_peak"], c["peak"],
                    c["tail_base"] + (i % c["tail_period"]) * np.float32(c["tail_step"])).astype(np.float32)


def test_softmax_wide_accumulator(kats):
    c = kats["softmax_wide_accumulator"]
    logits = peaked_logits(c)
    exps = np.exp(logits - logits.max()).astype(np.float32)
    sum64 = exps.astype(np.float64).sum()
    ref = (exps.astype(np.float64) / sum64).astype(np.float32)
    got = oracle.softmax(logits)
    rel = np.abs(got - ref) / np.maximum(np.abs(ref), 1e-9)
    assert rel.max() < c["tol"]
    # the f32-accumulator regression the reference guards against stays detectable
    s32 = np.float32(0)
    for e in exps:
        s32 = np.float32(s32 + e)
    regressed = np.abs(exps * np.float32(1.0 / s32) - ref) / np.maximum(np.abs(ref), 1e-9)
    assert regressed.max() > c["tol"]


def test_rmsnorm_kats(kats):
    for case in kats["rmsnorm"]:
        out = oracle.rmsnorm(case["x"], case["gain"], case["eps"])
        if "out" in case:
            assert np.array_equal(out, np.array(case["out"], np.float32)), case["src"]
        else:
            s = np.float32(1.0) / np.sqrt(np.float32(case["scale_is_inv_sqrt_of"]))
            assert abs(out[0] - s) < case["tol"] and abs(out[3] - 4 * s) < case["tol"]
            assert abs(float((out.astype(np.float32) ** 2).sum() / 4) - 1) < case["mean_square_tol"]


def test_rmsnorm_wide_accumulator(kats):
    c = kats["rmsnorm_wide_accumulator"]
    i = np.arange(c["n"])
    x = np.where(i < c["n_big"], c["big"],
                 np.float32(c["small_scale"]) * ((i % c["small_period"]).astype(np.float32) - np.float32(c["small_offset"]))).astype(np.float32)
    ss64 = (x.astype(np.float64) ** 2).sum()
    scale64 = 1.0 / math.sqrt(ss64 / c["n"] + float(np.float32(c["eps"])))
    ref = (x.astype(np.float64) * scale64).astype(np.float32)
    got = oracle.rmsnorm(x, np.ones_like(x), c["eps"])
    rel = np.abs(got - ref) / np.maximum(np.abs(ref), 1e-6)
    assert rel.max() < c["tol"]


def test_rope_kats(kats):
    fn = {"cos1": math.cos(1.0), "sin1": math.sin(1.0), "zero": 0.0}
    for case in kats["rope"]:
        out = oracle.rope_neox(case["x"], case["pos"], case["base"])
        if "out" in case:
            assert np.array_equal(out, np.array(case["out"], np.float32)), case["src"]
        else:
            want = np.array([fn[f] for f in case["out_fn"]], np.float32)
            assert np.abs(out - want).max() < case["tol"], case["src"]
            for j, f in enumerate(case["out_fn"]):
                if f == "zero":
                    assert out[j] == 0.0
    c = kats["rope_norm"]
    x = np.array(c["x"], np.float32)
    y = oracle.rope_neox(x, c["pos"], c["base"])
    assert abs(float((x * x).sum()) - float((y * y).sum())) < c["tol"]


def test_cache_kat(kats):
    c = kats["cache"]
    cache = oracle.Cache(c["n_layers"], c["kv_dim"])
    for l in c["layers_filled"]:
        cache.k[l] = np.full((c["fill_positions"], c["kv_dim"]), 1.0, np.float32)
        cache.v[l] = np.full((c["fill_positions"], c["kv_dim"]), 2.0, np.float32)
    assert cache.kv_len() == c["kv_len_before"]
    cache.evict_front(c["evict"])
    assert cache.kv_len() == c["kv_len_after"]
    assert cache.k[2].shape[0] == 2 and cache.v[6].shape[0] == 2
    assert cache.k[0].shape[0] == 0


def test_dot_kats(kats):
    c = kats["dot"]
    assert oracle.dot(c["basic"]["a"], c["basic"]["b"]) == c["basic"]["out"]
    assert oracle.dot([], []) == 0.0
    for n in c["lengths"]:
        a = (np.arange(n) * np.float32(0.1) - 1).astype(np.float32)
        b = (((np.arange(n) % 5).astype(np.float32) - 2) * np.float32(0.3)).astype(np.float32)
        want = np.float32(0)
        for x, y in zip(a, b):
            want = np.float32(want + np.float32(x * y))
        got = oracle.dot(a, b)
        assert abs(got - want) <= c["rel_tol"] * max(abs(want), 1.0), n


def test_prefill_equals_per_token(kats):
    """src/model.rs:672-708: batched prefill is bit-identical to per-token decode."""
    H, KVH, D = 32, 8, 64
    t = 9
    q = oracle.normal(1, (t, H * D))
    k = oracle.normal(2, (t, KVH * D))
    v = oracle.normal(3, (t, KVH * D))
    qg = oracle.normal(4, (D,), 1.0, 0.02)
    kg = oracle.normal(5, (D,), 1.0, 0.02)
    out_b, ck, cv, _, _ = oracle.attn_batch(q, k, v, 0, qg, kg, 1e6, 1e-5, H, KVH, D)
    cache = oracle.Cache(1, KVH * D)
    for i in range(t):
        o = cache.attn_step(0, q[i], k[i], v[i], qg, kg, 1e6, 1e-5, H, KVH, D, pos=i)
        assert np.array_equal(o, out_b[i])
    assert np.array_equal(cache.k[0], ck) and np.array_equal(cache.v[0], cv)
    # the multi-threaded harness changes nothing
    out_mt, _, _, _, _ = oracle.attn_batch(q, k, v, 0, qg, kg, 1e6, 1e-5, H, KVH, D, n_threads=4)
    assert np.array_equal(out_mt, out_b)


def test_prng_is_deterministic():
    a = oracle.normal(123, (1000,))
    b = oracle.normal(123, (1000,))
    assert np.array_equal(a, b)
    assert abs(float(a.mean())) < 0.1 and abs(float(a.std()) - 1) < 0.1
