"""Parity of the CUDA path (through the C-ABI) with the CPU oracle on seeded inputs.

Tolerances (stated by the hot-path contract): fp32 decode max |err| <= 1e-3;
kernel 1 (norm + RoPE) is compared at 2e-5 abs — its only rounding differences
from the reference are sinf/cosf ulps.
"""
import math

import numpy as np
import pytest

import bebelm_b200 as bb
import oracle

pytestmark = pytest.mark.gpu

H, KVH, D = 32, 8, 64
HID, KVD = H * D, KVH * D
DECODE_ATOL = 1e-3
ROPE_ATOL = 2e-5


def gains(seed):
    return oracle.normal(seed, (D,), 1.0, 0.02), oracle.normal(seed + 1, (D,), 1.0, 0.02)


# ------------------------------------------------------------- reference KATs --
def test_attention_kats(kats):
    for case in kats["attention"]:
        out = bb.attention_decode(case["q"], case["k"], case["v"], case["n_ctx"], case["n_heads"],
                                  case["n_kv_heads"], case["head_dim"])
        want = np.array(case["out"], np.float32)
        if case.get("exact"):
            assert np.array_equal(out, want), (case["src"], out)
        else:
            assert np.abs(out - want).max() < case["tol"], (case["src"], out)


def test_rmsnorm_kats_through_norm_rope(kats):
    # at pos 0 the rotation is the identity (sin 0 = 0, cos 0 = 1), so the fused kernel
    # must reproduce the rmsnorm known answers exactly
    for case in kats["rmsnorm"]:
        out = bb.norm_rope_heads(case["x"], 1, len(case["x"]), case["gain"], 0, 5e6, case["eps"])
        if "out" in case:
            assert np.array_equal(out, np.array(case["out"], np.float32)), case["src"]
        else:
            s = np.float32(1.0) / np.sqrt(np.float32(case["scale_is_inv_sqrt_of"]))
            assert abs(out[0] - s) < case["tol"] and abs(out[3] - 4 * s) < case["tol"]


def test_rope_kats_through_norm_rope(kats):
    for case in kats["rope"] + [kats["rope_norm"]]:
        x = np.array(case["x"], np.float32)
        g = np.ones_like(x)
        got = bb.norm_rope_heads(x, 1, x.size, g, case["pos"], case["base"], 1e-5)
        want = oracle.norm_rope_heads(x, 1, x.size, g, case["pos"], case["base"], 1e-5)
        assert np.abs(got - want).max() <= ROPE_ATOL, case["src"]


def test_empty_context_is_zero():
    out = bb.attention_decode(np.ones(HID, np.float32), np.zeros(0), np.zeros(0), 0, H, KVH, D)
    assert not out.any()


# ----------------------------------------------------------- kernel 1 parity --
@pytest.mark.parametrize("theta", [1e6, 5e6])
@pytest.mark.parametrize("pos0", [0, 511, 32767, 1_000_000])
def test_norm_rope_matches_oracle(theta, pos0):
    T = 17
    x = oracle.normal(11 + pos0, (T, H, D))
    g, _ = gains(7)
    got = bb.norm_rope_heads(x, H, D, g, pos0, theta, 1e-5, n_tokens=T).reshape(T, H, D)
    want = np.stack([oracle.norm_rope_heads(x[i], H, D, g, pos0 + i, theta, 1e-5).reshape(H, D) for i in range(T)])
    err = np.abs(got - want).max()
    assert err <= ROPE_ATOL, err
    # the norm itself (pos 0, identity rotation) is bit-exact
    if pos0 == 0:
        assert np.array_equal(got[0], want[0])


def test_softmax_wide_accumulator_through_attention(kats):
    """softmax.rs:59-108 discriminator as an attention problem: 4096 peaked scores."""
    c = kats["softmax_wide_accumulator"]
    i = np.arange(c["n"])
    logits = np.where(i < c["n_peak"], c["peak"],
                      c["tail_base"] + (i % c["tail_period"]) * np.float32(c["tail_step"])).astype(np.float32)
    q = np.zeros(D, np.float32)
    q[0] = 8.0                               # 8 * logit * 0.125 == logit exactly
    k = np.zeros((c["n"], D), np.float32)
    k[:, 0] = logits
    v = oracle.normal(5, (c["n"], D))
    got = bb.attention_decode(q, k, v, c["n"], 1, 1, D)
    want = oracle.attention_decode(q, k, v, c["n"], 1, 1, D)
    # f64 ground truth; the reference's own output accumulation (out += w*v in f32,
    # attention.rs:48-53) carries ~1e-6 of rounding on this case
    e = np.exp(logits.astype(np.float64) - logits.max())
    exact = (e / e.sum()) @ v.astype(np.float64)
    # an f32 running sum of the exps (the regression softmax.rs guards against) would
    # shift every output by ~1e-4 relative
    s32 = np.float32(0)
    for x in np.exp(logits - logits.max()).astype(np.float32):
        s32 = np.float32(s32 + x)
    regressed = np.abs((e @ v.astype(np.float64)) / np.float64(s32) - exact).max()
    assert np.abs(want - exact).max() < 1e-5
    assert np.abs(got - exact).max() < 1e-5 < regressed


@pytest.mark.parametrize("group", [1, 2, 3, 4, 8])
def test_gqa_groups_drop_in(group):
    n_kv = 2
    n_heads = group * n_kv
    n_ctx = 700
    q = oracle.normal(1, (n_heads * D,))
    k = oracle.normal(2, (n_ctx * n_kv * D,))
    v = oracle.normal(3, (n_ctx * n_kv * D,))
    got = bb.attention_decode(q, k, v, n_ctx, n_heads, n_kv, D)
    want = oracle.attention_decode(q, k, v, n_ctx, n_heads, n_kv, D)
    assert np.abs(got - want).max() <= DECODE_ATOL
    assert np.abs(got - want).max() <= 1e-5


@pytest.mark.parametrize("head_dim", [2, 8, 48])
def test_small_head_dims_drop_in(head_dim):
    q = oracle.normal(4, (4 * head_dim,))
    k = oracle.normal(5, (33 * 2 * head_dim,))
    v = oracle.normal(6, (33 * 2 * head_dim,))
    got = bb.attention_decode(q, k, v, 33, 4, 2, head_dim)
    want = oracle.attention_decode(q, k, v, 33, 4, 2, head_dim)
    assert np.abs(got - want).max() <= 1e-5


# ------------------------------------------------------- fused decode parity --
def _seed_cache(ndev, nref, layer, n, seed):
    k = oracle.normal(seed, (n, KVD))
    v = oracle.normal(seed + 1, (n, KVD))
    if n:
        ndev.append(layer, k, v)
    nref.append(layer, k, v)


def test_config1_decode_step():
    """Config 1: 512 cached positions, one step at pos 512, theta 1e6."""
    dev = bb.Cache(n_layers=1, max_context=4096)
    ref = oracle.Cache(1, KVD)
    _seed_cache(dev, ref, 0, 512, 100)
    qg, kg = gains(200)
    q, k, v = oracle.normal(1, (HID,)), oracle.normal(2, (KVD,)), oracle.normal(3, (KVD,))
    got = dev.attn_step(0, q, k, v, qg, kg, pos=512, theta=1e6)
    want = ref.attn_step(0, q, k, v, qg, kg, 1e6, 1e-5, H, KVH, D, pos=512)
    assert np.abs(got - want).max() <= DECODE_ATOL
    kd, vd = dev.read(0)
    assert kd.shape == (513, KVD)
    assert np.abs(kd - ref.k[0]).max() <= ROPE_ATOL and np.array_equal(vd, ref.v[0])


def test_config3_long_window_with_eviction():
    """Config 3 shape: a full 32768 window, steps that append one and evict the oldest."""
    n = 32768
    dev = bb.Cache(n_layers=1, max_context=n)
    ref = oracle.Cache(1, KVD)
    for c0 in range(0, n, 8192):
        _seed_cache(dev, ref, 0, 8192, 1000 + c0)
    qg, kg = gains(300)
    for step in range(3):
        pos = n + step
        q, k, v = oracle.normal(10 + step, (HID,)), oracle.normal(20 + step, (KVD,)), oracle.normal(30 + step, (KVD,))
        got = dev.attn_step(0, q, k, v, qg, kg, pos=pos, theta=1e6)
        want = ref.attn_step(0, q, k, v, qg, kg, 1e6, 1e-5, H, KVH, D, pos=pos)
        assert np.abs(got - want).max() <= DECODE_ATOL, step
        dev.evict_front(1)
        ref.evict_front(1)
        assert dev.kv_len() == ref.kv_len() == n


def test_window_bookkeeping_matches_reference_cache():
    """Appends and evictions of uneven sizes over several layers (src/cache.rs:40-48 rules)."""
    rng = np.random.default_rng(0)
    L = 3
    dev = bb.Cache(n_layers=L, max_context=300)
    ref = oracle.Cache(L, KVD)
    seed = 0
    for it in range(40):
        layer = int(rng.integers(0, L))
        if rng.random() < 0.6 or ref.kv_len() == 0:
            t = int(rng.integers(1, 90))
            if ref.k[layer].shape[0] + t > 300:
                continue
            seed += 2
            _seed_cache(dev, ref, layer, t, seed)
        else:
            nev = int(rng.integers(1, 120))
            dev.evict_front(nev)
            ref.evict_front(nev)
        assert dev.kv_len() == ref.kv_len()
        for l in range(L):
            kd, vd = dev.read(l)
            assert np.array_equal(kd, ref.k[l]) and np.array_equal(vd, ref.v[l]), (it, l)


def test_capacity_error_and_recovery():
    # max_context 128 -> a ring of ceil(128/64) + 2 = 4 pages: at least max_context + 64
    # positions always fit, up to 256 when the window starts on a page boundary
    dev = bb.Cache(n_layers=1, max_context=128)
    k = np.zeros((256, KVD), np.float32)
    dev.append(0, k, k)
    with pytest.raises(bb.BebelmError) as e:
        dev.append(0, k[:1], k[:1])
    assert e.value.code == bb.ERR_CAPACITY
    assert dev.kv_len() == 256  # a refused append changes nothing
    dev.evict_front(64)
    dev.append(0, k[:64], k[:64])
    assert dev.kv_len() == 256


def test_clone_forks_and_clear_resets():
    dev = bb.Cache(n_layers=2, max_context=1024)
    ref = oracle.Cache(2, KVD)
    for l in range(2):
        _seed_cache(dev, ref, l, 300, 50 + l)
    fork = dev.clone()
    ref_fork = ref.clone()
    qg, kg = gains(9)
    q, k, v = oracle.normal(1, (HID,)), oracle.normal(2, (KVD,)), oracle.normal(3, (KVD,))
    a = dev.attn_step(1, q, k, v, qg, kg, pos=300)
    b = ref.attn_step(1, q, k, v, qg, kg, 5e6, 1e-5, H, KVH, D, pos=300)
    assert np.abs(a - b).max() <= DECODE_ATOL
    assert fork.layer_len(1) == 300 and dev.layer_len(1) == 301  # the fork did not see the step
    q2 = oracle.normal(4, (HID,))
    c = fork.attn_step(1, q2, k, v, qg, kg, pos=300)
    d = ref_fork.attn_step(1, q2, k, v, qg, kg, 5e6, 1e-5, H, KVH, D, pos=300)
    assert np.abs(c - d).max() <= DECODE_ATOL
    dev.clear()
    assert dev.kv_len() == 0 and dev.pos == 0 and fork.kv_len() == 301


def test_batched_decode_across_sequences():
    lens = [1, 63, 64, 65, 700, 2049, 4100, 0]
    pool = bb.Pool(n_layers=1, n_pages=400)
    devs = [bb.Cache(max_context=8192, pool=pool) for _ in lens]
    refs = [oracle.Cache(1, KVD) for _ in lens]
    for i, n in enumerate(lens):
        _seed_cache(devs[i], refs[i], 0, n, 500 + 3 * i)
    qg, kg = gains(11)
    n = len(lens)
    q, k, v = oracle.normal(1, (n, HID)), oracle.normal(2, (n, KVD)), oracle.normal(3, (n, KVD))
    pos = [l + 7 for l in lens]
    got = bb.attn_decode_batched(devs, 0, q, k, v, qg, kg, pos, theta=1e6)
    for i in range(n):
        want = refs[i].attn_step(0, q[i], k[i], v[i], qg, kg, 1e6, 1e-5, H, KVH, D, pos=pos[i])
        assert np.abs(got[i] - want).max() <= DECODE_ATOL, i


def test_device_pointers_and_stream():
    torch = pytest.importorskip("torch")
    dev = bb.Cache(n_layers=1, max_context=2048)
    ref = oracle.Cache(1, KVD)
    _seed_cache(dev, ref, 0, 1000, 77)
    qg, kg = gains(13)
    q, k, v = oracle.normal(1, (HID,)), oracle.normal(2, (KVD,)), oracle.normal(3, (KVD,))
    s = torch.cuda.Stream()
    tq, tk, tv, tqg, tkg = (torch.from_numpy(x).cuda() for x in (q, k, v, qg, kg))
    torch.cuda.synchronize()
    with torch.cuda.stream(s):
        out = dev.attn_step(0, tq, tk, tv, tqg, tkg, pos=1000, stream=s)
    s.synchronize()
    want = ref.attn_step(0, q, k, v, qg, kg, 5e6, 1e-5, H, KVH, D, pos=1000)
    assert np.abs(out.cpu().numpy() - want).max() <= DECODE_ATOL


# -------------------------------------------------------------- prefill parity --
def test_prefill_chunks_match_oracle():
    """src/model.rs:232-254 with a second chunk on top of the first (absorb's 512-chunks)."""
    dev = bb.Cache(n_layers=1, max_context=4096)
    qg, kg = gains(21)
    outs, ref_cache_k, ref_cache_v = [], None, None
    for chunk, (pos0, t) in enumerate([(0, 300), (300, 212)]):
        q, k, v = oracle.normal(40 + chunk, (t, HID)), oracle.normal(50 + chunk, (t, KVD)), oracle.normal(60 + chunk, (t, KVD))
        got = dev.attn_prefill(0, q, k, v, qg, kg, pos0, theta=1e6)
        want, ref_cache_k, ref_cache_v, _, _ = oracle.attn_batch(q, k, v, pos0, qg, kg, 1e6, 1e-5, H, KVH, D,
                                                                  ref_cache_k, ref_cache_v, n_threads=oracle.max_threads())
        assert np.abs(got - want).max() <= DECODE_ATOL, chunk
    kd, vd = dev.read(0)
    assert np.abs(kd - ref_cache_k).max() <= ROPE_ATOL and np.array_equal(vd, ref_cache_v)


def test_prefill_equals_per_token_decode():
    """src/model.rs:672-708 analogue: prefill == token-by-token attn_step (to fp32 tolerance)."""
    t = 130
    qg, kg = gains(31)
    q, k, v = oracle.normal(1, (t, HID)), oracle.normal(2, (t, KVD)), oracle.normal(3, (t, KVD))
    a = bb.Cache(n_layers=1, max_context=1024)
    b = bb.Cache(n_layers=1, max_context=1024)
    pre = a.attn_prefill(0, q, k, v, qg, kg, 0)
    step = np.stack([b.attn_step(0, q[i], k[i], v[i], qg, kg, pos=i) for i in range(t)])
    assert np.abs(pre - step).max() <= 1e-5
    ka, va = a.read(0)
    kb, vb = b.read(0)
    assert np.array_equal(ka, kb) and np.array_equal(va, vb)


def test_config2_prefill_2048():
    """Config 2: 2048 tokens into an empty cache, theta 1e6."""
    t = 2048
    qg, kg = gains(41)
    q, k, v = oracle.normal(1, (t, HID)), oracle.normal(2, (t, KVD)), oracle.normal(3, (t, KVD))
    dev = bb.Cache(n_layers=1, max_context=t)
    got = dev.attn_prefill(0, q, k, v, qg, kg, 0, theta=1e6)
    want, _, _, _, _ = oracle.attn_batch(q, k, v, 0, qg, kg, 1e6, 1e-5, H, KVH, D, n_threads=oracle.max_threads())
    assert np.abs(got - want).max() <= DECODE_ATOL


# ------------------------------------------------ tensor-core prefill (bf16) --
PREFILL_REL = 2e-2  # bf16 operands, fp32 accumulation: max |err| / max |want|


def _bf16_round(x):
    torch = pytest.importorskip("torch")
    return torch.from_numpy(np.ascontiguousarray(x)).to(torch.bfloat16).float().numpy()


def _prefill_bf16(dev_cache, q, k, v, qg, kg, pos0, theta):
    torch = pytest.importorskip("torch")
    tq, tk, tv = (torch.from_numpy(np.ascontiguousarray(x)).cuda().to(torch.bfloat16) for x in (q, k, v))
    tqg, tkg = torch.from_numpy(qg).cuda(), torch.from_numpy(kg).cuda()
    out = dev_cache.attn_prefill(0, tq, tk, tv, tqg, tkg, pos0, theta=theta)
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("t", [128, 300, 1000])
def test_tensor_core_prefill_matches_oracle(t):
    qg, kg = gains(61)
    q, k, v = (_bf16_round(oracle.normal(s, shp)) for s, shp in ((1, (t, HID)), (2, (t, KVD)), (3, (t, KVD))))
    dev = bb.Cache(n_layers=1, max_context=4096)
    got = _prefill_bf16(dev, q, k, v, qg, kg, 0, 1e6)
    want = oracle.attn_batch(q, k, v, 0, qg, kg, 1e6, 1e-5, H, KVH, D, n_threads=oracle.max_threads())[0]
    rel = np.abs(got - want).max() / np.abs(want).max()
    assert rel <= PREFILL_REL, rel
    # the cache holds the fp32 normed/roped keys and raw values either way
    kd, vd = dev.read(0)
    ck = oracle.attn_batch(q, k, v, 0, qg, kg, 1e6, 1e-5, H, KVH, D)[1]
    assert np.abs(kd - ck).max() <= ROPE_ATOL and np.array_equal(vd, v)


@pytest.mark.parametrize("t", [300, 2048])
def test_f32_inputs_on_tensor_cores_match_oracle(t):
    """BEBELM_F32_TENSOR: the fp32 inputs a Rust attn_batch passes (host memory, not
    bf16-rounded), normed and roped in fp32, attention on the tensor cores."""
    qg, kg = gains(63)
    q, k, v = oracle.normal(31, (t, HID)), oracle.normal(32, (t, KVD)), oracle.normal(33, (t, KVD))
    dev = bb.Cache(n_layers=1, max_context=4096)
    got = dev.attn_prefill(0, q, k, v, qg, kg, 0, theta=1e6, tensor_cores=True)
    want, ck, cv, _, _ = oracle.attn_batch(q, k, v, 0, qg, kg, 1e6, 1e-5, H, KVH, D, n_threads=oracle.max_threads())
    rel = np.abs(got - want).max() / np.abs(want).max()
    assert rel <= PREFILL_REL, rel
    # the cache holds exactly what the fp32 path stores
    kd, vd = dev.read(0)
    assert np.abs(kd - ck).max() <= ROPE_ATOL and np.array_equal(vd, v)


def test_tensor_core_prefill_on_a_cached_prefix():
    """A chunk after 333 cached positions (not a multiple of the 128-key tile), after eviction."""
    qg, kg = gains(71)
    dev = bb.Cache(n_layers=1, max_context=4096)
    pk, pv = oracle.normal(5, (400, KVD)), oracle.normal(6, (400, KVD))
    dev.append(0, pk, pv)
    dev.evict_front(67)
    t = 257
    q, k, v = (_bf16_round(oracle.normal(s, shp)) for s, shp in ((7, (t, HID)), (8, (t, KVD)), (9, (t, KVD))))
    got = _prefill_bf16(dev, q, k, v, qg, kg, 400, 5e6)
    want = oracle.attn_batch(q, k, v, 400, qg, kg, 5e6, 1e-5, H, KVH, D, pk[67:], pv[67:],
                             n_threads=oracle.max_threads())[0]
    rel = np.abs(got - want).max() / np.abs(want).max()
    assert rel <= PREFILL_REL, rel


def test_config2_tensor_core_prefill_2048():
    t = 2048
    qg, kg = gains(81)
    q, k, v = (_bf16_round(oracle.normal(s, shp)) for s, shp in ((11, (t, HID)), (12, (t, KVD)), (13, (t, KVD))))
    dev = bb.Cache(n_layers=1, max_context=t)
    got = _prefill_bf16(dev, q, k, v, qg, kg, 0, 1e6)
    want = oracle.attn_batch(q, k, v, 0, qg, kg, 1e6, 1e-5, H, KVH, D, n_threads=oracle.max_threads())[0]
    rel = np.abs(got - want).max() / np.abs(want).max()
    assert rel <= PREFILL_REL, rel


# ------------------------------------------------------------ bf16 KV cache --
def _bf16(x):
    torch = pytest.importorskip("torch")
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(torch.bfloat16).float().numpy()


def test_bf16_cache_decode_matches_oracle_on_the_same_values():
    """Over bf16-exact K/V the bf16 cache must give what the fp32 reference arithmetic gives."""
    n = 3000
    dev = bb.Cache(n_layers=2, max_context=4096, kv_dtype=bb.BF16)
    k, v = _bf16(oracle.normal(1, (n, KVD))), _bf16(oracle.normal(2, (n, KVD)))
    dev.append(1, k, v)
    dev.evict_front(129)
    kd, vd = dev.read(1)
    assert np.array_equal(kd, k[129:]) and np.array_equal(vd, v[129:])
    torch = pytest.importorskip("torch")
    q = oracle.normal(3, (HID,))
    got = dev.decode(1, torch.from_numpy(q).cuda()).cpu().numpy()
    want = oracle.attention_decode(q, k[129:], v[129:], n - 129, H, KVH, D)
    assert np.abs(got - want).max() <= 1e-5


def _ref_step_bf16(ref, q, k, v, qg, kg, pos):
    """attn_step on the oracle, with the appended k and v rounded to bf16 as the bf16 cache stores them."""
    qn = oracle.norm_rope_heads(q, H, D, qg, pos, 1e6, 1e-5)
    kn = _bf16(oracle.norm_rope_heads(k, KVH, D, kg, pos, 1e6, 1e-5))
    ref.append(0, kn, _bf16(v))
    return oracle.attention_decode(qn, ref.k[0], ref.v[0], ref.k[0].shape[0], H, KVH, D)


def test_bf16_cache_fused_step_and_batched():
    qg, kg = gains(91)
    dev = bb.Cache(n_layers=1, max_context=2048, kv_dtype=bb.BF16)
    ref = oracle.Cache(1, KVD)
    k0, v0 = _bf16(oracle.normal(4, (700, KVD))), _bf16(oracle.normal(5, (700, KVD)))
    dev.append(0, k0, v0)
    ref.append(0, k0, v0)
    for step in range(3):
        q, k, v = oracle.normal(10 + step, (HID,)), oracle.normal(20 + step, (KVD,)), oracle.normal(30 + step, (KVD,))
        got = dev.attn_step(0, q, k, v, qg, kg, pos=700 + step, theta=1e6)
        want = _ref_step_bf16(ref, q, k, v, qg, kg, 700 + step)
        assert np.abs(got - want).max() <= 1e-4, step
    kd, vd = dev.read(0)
    # the appended k may differ by one bf16 ulp where sinf/cosf ulps move it across a rounding boundary
    assert np.abs(kd - ref.k[0]).max() <= 2e-2 and np.array_equal(vd, ref.v[0])
    pool = bb.Pool(n_layers=1, n_pages=100, kv_dtype=bb.BF16)
    lens = [5, 130, 1000]
    devs = [bb.Cache(max_context=2048, pool=pool, kv_dtype=bb.BF16) for _ in lens]
    refs = [oracle.Cache(1, KVD) for _ in lens]
    for i, n in enumerate(lens):
        kk, vv = _bf16(oracle.normal(40 + i, (n, KVD))), _bf16(oracle.normal(50 + i, (n, KVD)))
        devs[i].append(0, kk, vv)
        refs[i].append(0, kk, vv)
    q, k, v = oracle.normal(6, (3, HID)), oracle.normal(7, (3, KVD)), oracle.normal(8, (3, KVD))
    got = bb.attn_decode_batched(devs, 0, q, k, v, qg, kg, [n for n in lens], theta=1e6)
    for i in range(3):
        want = _ref_step_bf16(refs[i], q[i], k[i], v[i], qg, kg, lens[i])
        assert np.abs(got[i] - want).max() <= 1e-4, i


def test_bf16_cache_tensor_core_prefill():
    qg, kg = gains(95)
    dev = bb.Cache(n_layers=1, max_context=4096, kv_dtype=bb.BF16)
    pk, pv = _bf16(oracle.normal(5, (300, KVD))), _bf16(oracle.normal(6, (300, KVD)))
    dev.append(0, pk, pv)
    t = 400
    q, k, v = (_bf16_round(oracle.normal(s, shp)) for s, shp in ((7, (t, HID)), (8, (t, KVD)), (9, (t, KVD))))
    got = _prefill_bf16(dev, q, k, v, qg, kg, 300, 1e6)
    want = oracle.attn_batch(q, k, v, 300, qg, kg, 1e6, 1e-5, H, KVH, D, pk, pv, n_threads=oracle.max_threads())[0]
    rel = np.abs(got - want).max() / np.abs(want).max()
    assert rel <= PREFILL_REL, rel


# ------------------------------------------------------------- fp8 KV cache --
def _fp8(x):
    """x rounded to e4m3 (nearest even; these N(0,1) values are far from the +-448 limit)."""
    torch = pytest.importorskip("torch")
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(torch.float8_e4m3fn).float().numpy()


def test_fp8_cache_decode_matches_oracle_on_the_same_values():
    """Over e4m3-exact K/V the fp8 cache must give what the fp32 reference arithmetic gives."""
    n = 3000
    dev = bb.Cache(n_layers=2, max_context=4096, kv_dtype=bb.FP8)
    k, v = _fp8(oracle.normal(1, (n, KVD))), _fp8(oracle.normal(2, (n, KVD)))
    dev.append(1, k, v)
    dev.evict_front(129)
    kd, vd = dev.read(1)
    assert np.array_equal(kd, k[129:]) and np.array_equal(vd, v[129:])
    torch = pytest.importorskip("torch")
    q = oracle.normal(3, (HID,))
    got = dev.decode(1, torch.from_numpy(q).cuda()).cpu().numpy()
    want = oracle.attention_decode(q, k[129:], v[129:], n - 129, H, KVH, D)
    assert np.abs(got - want).max() <= 1e-5


FP8_VS_FP32_ATOL = 5e-2  # fp8 cache against the fp32 reference on unrounded N(0,1) K/V


def test_fp8_cache_accuracy_against_fp32_reference():
    """The stated cost of the fp8 cache: on N(0,1) data (4096 positions) the decode output stays
    within FP8_VS_FP32_ATOL of the fp32 reference on the unrounded values."""
    torch = pytest.importorskip("torch")
    n = 4096
    dev = bb.Cache(n_layers=1, max_context=n, kv_dtype=bb.FP8)
    k, v = oracle.normal(61, (n, KVD)), oracle.normal(62, (n, KVD))
    dev.append(0, k, v)
    q = oracle.normal(63, (HID,))
    got = dev.decode(0, torch.from_numpy(q).cuda()).cpu().numpy()
    want = oracle.attention_decode(q, k, v, n, H, KVH, D)
    err = np.abs(got - want).max()
    print(f"fp8 cache vs fp32 reference: max |err| {err:.3e} (outputs up to {np.abs(want).max():.3f})")
    assert err <= FP8_VS_FP32_ATOL, err


def test_fp8_cache_fused_step_and_batched():
    """The fused step and batched decode on an fp8 cache. The oracle step appends the k the
    cache holds (read back: the device's RoPE may round one element to the next e4m3 value)."""
    torch = pytest.importorskip("torch")
    qg, kg = gains(93)
    dev = bb.Cache(n_layers=1, max_context=2048, kv_dtype=bb.FP8)
    ref = oracle.Cache(1, KVD)
    k0, v0 = _fp8(oracle.normal(4, (700, KVD))), _fp8(oracle.normal(5, (700, KVD)))
    dev.append(0, k0, v0)
    ref.append(0, k0, v0)
    for step in range(3):
        q, k, v = oracle.normal(10 + step, (HID,)), oracle.normal(20 + step, (KVD,)), oracle.normal(30 + step, (KVD,))
        got = dev.attn_step(0, q, k, v, qg, kg, pos=700 + step, theta=1e6)
        kd, vd = dev.read(0)
        kn = oracle.norm_rope_heads(k, KVH, D, kg, 700 + step, 1e6, 1e-5)
        # the stored k is the e4m3 rounding of the normed, roped k (one step apart at most)
        assert np.abs(kd[-1] - kn).max() <= 0.07 * np.abs(kn).max() + 1e-6
        assert np.array_equal(vd[-1], _fp8(v))
        ref.append(0, kd[-1], vd[-1])
        qn = oracle.norm_rope_heads(q, H, D, qg, 700 + step, 1e6, 1e-5)
        want = oracle.attention_decode(qn, ref.k[0], ref.v[0], ref.k[0].shape[0], H, KVH, D)
        assert np.abs(got - want).max() <= 1e-4, step
    pool = bb.Pool(n_layers=1, n_pages=100, kv_dtype=bb.FP8)
    lens = [5, 130, 1000]
    devs = [bb.Cache(max_context=2048, pool=pool, kv_dtype=bb.FP8) for _ in lens]
    refs = [oracle.Cache(1, KVD) for _ in lens]
    for i, n in enumerate(lens):
        kk, vv = _fp8(oracle.normal(40 + i, (n, KVD))), _fp8(oracle.normal(50 + i, (n, KVD)))
        devs[i].append(0, kk, vv)
        refs[i].append(0, kk, vv)
    q, k, v = oracle.normal(6, (3, HID)), oracle.normal(7, (3, KVD)), oracle.normal(8, (3, KVD))
    got = bb.attn_decode_batched(devs, 0, q, k, v, qg, kg, [n for n in lens], theta=1e6)
    for i in range(3):
        kd, vd = devs[i].read(0)
        refs[i].append(0, kd[-1], vd[-1])
        qn = oracle.norm_rope_heads(q[i], H, D, qg, lens[i], 1e6, 1e-5)
        want = oracle.attention_decode(qn, refs[i].k[0], refs[i].v[0], refs[i].k[0].shape[0], H, KVH, D)
        assert np.abs(got[i] - want).max() <= 1e-4, i


def test_fp8_cache_tensor_core_prefill():
    """A bf16 chunk on top of an fp8 prefix: the prefix enters the tensor cores as the cache
    holds it; the chunk's own keys as bf16 (the cache stores their e4m3 rounding)."""
    qg, kg = gains(97)
    dev = bb.Cache(n_layers=1, max_context=4096, kv_dtype=bb.FP8)
    pk, pv = _fp8(oracle.normal(5, (300, KVD))), _fp8(oracle.normal(6, (300, KVD)))
    dev.append(0, pk, pv)
    t = 400
    q, k, v = (_bf16_round(oracle.normal(s, shp)) for s, shp in ((7, (t, HID)), (8, (t, KVD)), (9, (t, KVD))))
    got = _prefill_bf16(dev, q, k, v, qg, kg, 300, 1e6)
    want = oracle.attn_batch(q, k, v, 300, qg, kg, 1e6, 1e-5, H, KVH, D, pk, pv, n_threads=oracle.max_threads())[0]
    rel = np.abs(got - want).max() / np.abs(want).max()
    assert rel <= PREFILL_REL, rel
    kd, vd = dev.read(0)
    assert np.array_equal(vd[300:], _fp8(v))
