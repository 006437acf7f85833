"""Parity of the benchmarked paths, run the way bench.py times them.

The bench's decode steps are device-pointer calls enqueued back to back on one stream with
no host synchronisation between them, so consecutive decode grids overlap through
programmatic dependent launch: a step norms and ropes its inputs and copies its first pages
before the previous grid has finished. These tests run exactly that (every step's output to a
row of its own) and only then compare every row with the oracle's sequence of
``attn_step`` calls (src/model.rs:440-451), plus the cache read back at the end:

* config 3: a full 32768-position window (fp32, bf16 and fp8 caches), 64 steps, each followed by
  evict_front(1);
* config 4 at its full shape: 64 sequences with lengths U[1024, 16384] (seed 4), 8 batched
  steps with the default split plan;
* the 8192-token tensor-core prefill (config 5's layer), on sampled query rows.

Tolerances: decode max |err| <= 1e-3; the cached k within 2e-5 (sinf/cosf ulps of the RoPE),
the cached v bit-exact; tensor-core prefill <= 2e-2 relative to max |out|.
"""
import numpy as np
import pytest

import bebelm_b200 as bb
import oracle

pytestmark = pytest.mark.gpu

H, KVH, D = 32, 8, 64
HID, KVD = H * D, KVH * D
THETA, EPS = 1e6, 1e-5
DECODE_ATOL = 1e-3
ROPE_ATOL = 2e-5
PREFILL_REL = 2e-2


def _gains(seed):
    return oracle.normal(seed, (D,), 1.0, 0.02), oracle.normal(seed + 1, (D,), 1.0, 0.02)


@pytest.mark.parametrize("kv_dtype", [bb.F32, bb.BF16, bb.FP8])
def test_config3_pdl_chained_steps_match_oracle(kv_dtype):
    torch = pytest.importorskip("torch")
    n, steps = 32768, 64
    dev = bb.Cache(n_layers=1, max_context=n, kv_dtype=kv_dtype)
    ref = oracle.Cache(1, KVD)
    narrow = {bb.BF16: torch.bfloat16, bb.FP8: torch.float8_e4m3fn}.get(kv_dtype)
    rnd = (lambda x: torch.from_numpy(x).to(narrow).float().numpy()) if narrow else (lambda x: x)
    for c0 in range(0, n, 8192):
        k, v = rnd(oracle.normal(3000 + c0, (8192, KVD))), rnd(oracle.normal(3001 + c0, (8192, KVD)))
        dev.append(0, k, v)
        ref.append(0, k, v)
    qg, kg = _gains(310)
    Qh, Kh, Vh = oracle.normal(41, (steps, HID)), oracle.normal(42, (steps, KVD)), oracle.normal(43, (steps, KVD))
    if narrow:
        Vh = rnd(Vh)
    Q, K, V = (torch.from_numpy(x).cuda() for x in (Qh, Kh, Vh))
    tqg, tkg = torch.from_numpy(qg).cuda(), torch.from_numpy(kg).cuda()
    OUT = torch.full((steps, HID), float("nan"), device="cuda")
    stream = torch.cuda.current_stream()
    torch.cuda.synchronize()
    # the bench's timed loop: no host synchronisation from the first step to the last
    for i in range(steps):
        dev.attn_step(0, Q[i], K[i], V[i], tqg, tkg, pos=n + i, theta=THETA, eps=EPS, out=OUT[i], stream=stream)
        dev.evict_front(1)
    dev.check(stream)
    got = OUT.cpu().numpy()
    threads = oracle.max_threads()
    kd, vd = dev.read(0)
    for i in range(steps):
        if narrow:
            # the oracle step appends exactly the k the cache holds (its bf16 / e4m3 rounding)
            kn = kd[n - steps + i]
            qn = oracle.norm_rope_heads(Qh[i], H, D, qg, n + i, THETA, EPS)
            ref.append(0, kn, Vh[i])
            want = oracle.attention_decode(qn, ref.k[0], ref.v[0], ref.k[0].shape[0], H, KVH, D, n_threads=threads)
        else:
            want = ref.attn_step(0, Qh[i], Kh[i], Vh[i], qg, kg, THETA, EPS, H, KVH, D, pos=n + i,
                                 n_threads=threads)
        ref.evict_front(1)
        err = np.abs(got[i] - want).max()
        assert err <= DECODE_ATOL, (i, err)
    assert dev.kv_len() == ref.kv_len() == n
    assert np.array_equal(vd, ref.v[0])
    assert np.abs(kd - ref.k[0]).max() <= ROPE_ATOL


def test_config4_full_shape_batched_steps_match_oracle():
    torch = pytest.importorskip("torch")
    steps = 8
    lengths = np.random.default_rng(4).integers(1024, 16385, size=64)
    n = len(lengths)
    pages = sum(int(l) // 64 + (steps + 72) // 64 + 3 for l in lengths)
    pool = bb.Pool(n_layers=1, n_pages=pages)
    devs = [bb.Cache(max_context=int(l) + steps + 72, pool=pool) for l in lengths]
    refs = [oracle.Cache(1, KVD) for _ in lengths]
    for i, l in enumerate(lengths):
        k, v = oracle.normal(7000 + 2 * i, (int(l), KVD)), oracle.normal(7001 + 2 * i, (int(l), KVD))
        devs[i].append(0, k, v)
        refs[i].append(0, k, v)
    qg, kg = _gains(410)
    Qh, Kh, Vh = (oracle.normal(50 + s, (steps, n, w)) for s, w in ((0, HID), (1, KVD), (2, KVD)))
    Q, K, V = (torch.from_numpy(x).cuda() for x in (Qh, Kh, Vh))
    tqg, tkg = torch.from_numpy(qg).cuda(), torch.from_numpy(kg).cuda()
    OUT = torch.full((steps, n, HID), float("nan"), device="cuda")
    stream = torch.cuda.current_stream()
    pos = [int(l) for l in lengths]
    torch.cuda.synchronize()
    for s in range(steps):  # the bench's loop, no host synchronisation between steps
        bb.attn_decode_batched(devs, 0, Q[s], K[s], V[s], tqg, tkg, pos, theta=THETA, out=OUT[s], stream=stream)
        pos = [p + 1 for p in pos]
    devs[0].check(stream)
    got = OUT.cpu().numpy()
    threads = oracle.max_threads()
    for s in range(steps):
        for i in range(n):
            want = refs[i].attn_step(0, Qh[s, i], Kh[s, i], Vh[s, i], qg, kg, THETA, EPS, H, KVH, D,
                                     pos=int(lengths[i]) + s, n_threads=threads)
            err = float(np.abs(got[s, i] - want).max())
            assert err <= DECODE_ATOL, (s, i, err)
    for i in (0, int(np.argmax(lengths)), n - 1):
        kd, vd = devs[i].read(0)
        assert np.array_equal(vd, refs[i].v[0]), i
        assert np.abs(kd - refs[i].k[0]).max() <= ROPE_ATOL, i
    for c in devs:
        c.close()
    pool.close()


def test_tensor_core_prefill_8192_matches_oracle_rows():
    """Config 5's layer: 8192 bf16 tokens into an empty cache. The oracle's per-token
    attention (src/model.rs:232-254: row i attends to keys 0..i) is evaluated on sampled
    rows: the first tile, every 61st row and the last tile."""
    torch = pytest.importorskip("torch")
    t = 8192
    qg, kg = _gains(91)

    def bf16(x):
        return torch.from_numpy(x).to(torch.bfloat16)

    q, k, v = (bf16(oracle.normal(s, shp)) for s, shp in ((21, (t, HID)), (22, (t, KVD)), (23, (t, KVD))))
    dev = bb.Cache(n_layers=1, max_context=t)
    out = dev.attn_prefill(0, q.cuda(), k.cuda(), v.cuda(), torch.from_numpy(qg).cuda(), torch.from_numpy(kg).cuda(),
                           0, theta=THETA)
    dev.check()
    got = out.cpu().numpy()
    qf, kf, vf = (x.float().numpy() for x in (q, k, v))
    # the cache holds the fp32 normed/roped keys (kernel 1) and the raw values
    kd, vd = dev.read(0)
    assert np.array_equal(vd, vf)
    kn = np.stack([oracle.norm_rope_heads(kf[i], KVH, D, kg, i, THETA, EPS) for i in range(t)])
    assert np.abs(kd - kn).max() <= ROPE_ATOL
    rows = sorted(set(range(0, 128)) | set(range(0, t, 61)) | set(range(t - 128, t)))
    threads = oracle.max_threads()
    want = np.stack([oracle.attention_decode(oracle.norm_rope_heads(qf[i], H, D, qg, i, THETA, EPS), kn[: i + 1],
                                             vf[: i + 1], i + 1, H, KVH, D, n_threads=threads) for i in rows])
    rel = np.abs(got[rows] - want).max() / np.abs(want).max()
    assert rel <= PREFILL_REL, rel
