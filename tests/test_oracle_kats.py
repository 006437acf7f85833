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


# ------------------------------------------------------------- quantized path --
def _patched(case, blocks=1):
    b = np.zeros(case["len"], np.uint8)
    for k, v in case["set"].items():
        b[int(k)] = v
    return np.tile(b, blocks)


def q4k_test_block():
    b = np.zeros(144, np.uint8)
    b[0:2] = [0x00, 0x3c]
    b[2:4] = [0x00, 0x34]
    b[4:16] = [(j * 17 + 5) & 255 for j in range(12)]
    b[16:144] = [(i * 37 + 11) & 255 for i in range(128)]
    return b, np.array([((i % 7) - 3) * 0.1 for i in range(256)], np.float32)


def q6k_test_block():
    b = np.zeros(210, np.uint8)
    b[208:210] = [0x00, 0x3c]
    b[0:128] = [(i * 53 + 17) & 255 for i in range(128)]
    b[128:192] = [(i * 97 + 5) & 255 for i in range(64)]
    b[192:208] = [(j * 29 + 3) & 255 for j in range(16)]
    return b, np.array([((i % 5) - 2) * 0.1 for i in range(256)], np.float32)


def test_quant_kats(kats):
    q = kats["quant"]
    for bits, val in q["f16"]["exact"]:
        got = oracle.f16_to_f32(bits)
        assert got == float(val) and math.copysign(1, got) == math.copysign(1, float(val)), (bits, got)
    assert all(math.isnan(oracle.f16_to_f32(b)) for b in q["f16"]["nan"])
    for bits, val, tol in q["f16"]["approx"]:
        assert abs(oracle.f16_to_f32(bits) - val) < tol
    for name, dtype in (("q4k_block", oracle.GG_Q4_K), ("q6k_block", oracle.GG_Q6_K)):
        out = oracle.dequantize(dtype, _patched(q[name]), 256)
        for i, v in q[name]["out"].items():
            assert out[int(i)] == v, (name, i, out[int(i)])
    f32 = np.array(q["dispatch_f32"]["values"], np.float32)
    assert np.array_equal(oracle.dequantize(oracle.GG_F32, f32.view(np.uint8), 3), f32)
    f16 = np.array(q["dispatch_f16"]["bits"], np.uint16).view(np.uint8)
    assert list(oracle.dequantize(oracle.GG_F16, f16, 4)) == q["dispatch_f16"]["out"]
    two = oracle.dequantize(oracle.GG_Q4_K, _patched(q["dispatch_two_q4k"], 2), 512)
    assert all(two[int(i)] == v for i, v in q["dispatch_two_q4k"]["out"].items())


def test_matvec_kats(kats):
    q = kats["quant"]
    c = q["matvec_f32_small"]
    w = np.array(c["w"], np.float32).view(np.uint8)
    for x, want in c["cases"]:
        assert list(oracle.matvec(oracle.GG_F32, w, c["n_in"], c["n_out"], x)) == want
    c = q["matvec_f16_small"]
    w = np.array(c["bits"], np.uint16).view(np.uint8)
    assert list(oracle.matvec(oracle.GG_F16, w, c["n_in"], c["n_out"], c["x"])) == c["out"]
    c = q["matvec_q4k_single_row"]
    x = np.zeros(256, np.float32)
    x[0] = 1.0
    assert oracle.matvec(oracle.GG_Q4_K, _patched(c), 256, 1, x)[0] == c["out"]
    # the Q8 path equals the exact dot of the dequantized weights with the Q8-rounded activations
    for (blk, x), dtype, name in ((q4k_test_block(), oracle.GG_Q4_K, "q4k_test_block"),
                                  (q6k_test_block(), oracle.GG_Q6_K, "q6k_test_block")):
        wts = oracle.dequantize(dtype, blk, 256)
        qx, sx, _ = oracle.quantize_q8(x)
        ref = np.float32(0)
        for wi, qi in zip(wts, qx):
            ref = np.float32(ref + np.float32(wi * np.float32(sx[0] * np.float32(qi))))
        y = oracle.matvec(dtype, blk, 256, 1, x)[0]
        assert abs(y - ref) <= q[name]["tol"] * max(abs(ref), 1.0), (name, y, ref)
    # rows are independent dots, bit for bit
    n_in, n_out = 40, 128
    w = np.array([((i % 13) - 6) * 0.05 for i in range(n_in * n_out)], np.float32)
    x = np.array([((i % 7) - 3) * 0.1 for i in range(n_in)], np.float32)
    y = oracle.matvec(oracle.GG_F32, w.view(np.uint8), n_in, n_out, x)
    for o in range(n_out):
        assert y[o] == oracle.dot(w[o * n_in:(o + 1) * n_in], x)


def test_matmul_is_matvec_per_token():
    rng = np.random.default_rng(3)
    blk = rng.integers(0, 256, size=8 * 144 * 4, dtype=np.uint8)
    blk.reshape(-1, 144)[:, 1] = 0x38  # d = 0.5
    blk.reshape(-1, 144)[:, 3] = 0x30  # dmin = 0.125
    x = rng.standard_normal((3, 2048)).astype(np.float32)
    y = oracle.matmul(oracle.GG_Q4_K, blk, 2048, 4, x, 3)
    for t in range(3):
        assert np.array_equal(y[t], oracle.matvec(oracle.GG_Q4_K, blk, 2048, 4, x[t]))


def test_sampler_kats(kats):
    """Greedy sampling (src/sampler.rs:64-88, argmax :139-149) against the reference's tests."""
    for c in kats["sampler"]:
        logits = np.array(c["logits"], np.float32)
        assert oracle.sample_greedy(logits, c["history"], c["repeat_penalty"]) == c["token"], c["src"]
    # the penalty rewrites the seen logits in place, each distinct token once
    logits = np.array([10.0, 4.0, -1.0], np.float32)
    oracle.sample_greedy(logits, [0, 0, 2], 2.0)
    assert list(logits) == [5.0, 4.0, -2.0]


def test_argmax_scan_semantics():
    """The reference's strict `>` scan from -inf: first index on ties, NaN never wins, and 0
    when nothing is above -inf."""
    nan, inf = float("nan"), float("inf")
    assert oracle.argmax([2.0, 5.0, 5.0, 1.0]) == 1
    assert oracle.argmax([nan, 1.0, nan, 3.0]) == 3
    assert oracle.argmax([-inf, -inf]) == 0
    assert oracle.argmax([nan, nan]) == 0
    assert oracle.argmax([-0.0, 0.0]) == 0
    assert oracle.argmax([-inf, -3.0]) == 1
