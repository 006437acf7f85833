"""The whole attention operator (src/model.rs:430-455 attn_step, 224-258 attn_batch) in one call.

The one-call forms must equal the composition of the pieces that are pinned on their own
(quantized projections: bit for bit with the oracle; the fused step / prefill: within their
tolerances) bit for bit, and the end-to-end result must match the oracle's composition. The
end-to-end tolerance is the attention's, carried through W_o: the output projection
re-quantizes the attention output to Q8, where a 1e-6 attention difference can move a value
across a rounding boundary (one quantum = max|a|/127).
"""
import numpy as np
import pytest

import bebelm_b200 as bb
import oracle
from test_gpu_quant import random_q4k, random_q6k

pytestmark = pytest.mark.gpu

H, KVH, D, HID = 32, 8, 64, 2048
KVD = KVH * D
THETA, EPS = 1e6, 1e-5


def _layer(seed=1):
    wq = random_q4k(HID, HID, seed)
    wk = random_q4k(KVD, HID, seed + 1)
    wv = random_q6k(KVD, HID, seed + 2)
    wo = random_q4k(HID, HID, seed + 3)
    qg, kg = (1 + 0.02 * oracle.normal(seed + s, D) for s in (4, 5))
    W = bb.AttnWeights((bb.GGML_Q4_K, wq), (bb.GGML_Q4_K, wk), (bb.GGML_Q6_K, wv), (bb.GGML_Q4_K, wo), qg, kg)
    return W, (wq, wk, wv, wo, qg, kg)


def _x(seed, shape):
    return (0.5 * oracle.normal(seed, shape)).astype(np.float32)


def test_layer_step_equals_its_pieces_and_the_oracle():
    W, (wq, wk, wv, wo, qg, kg) = _layer()
    a = bb.Cache(n_layers=2, max_context=512)
    pre_k, pre_v = oracle.normal(11, (100, KVD)), oracle.normal(12, (100, KVD))
    a.append(1, pre_k, pre_v)
    b = a.clone()
    ref = oracle.Cache(2, KVD)
    ref.k[1], ref.v[1] = pre_k.copy(), pre_v.copy()
    for i in range(6):
        x = _x(20 + i, HID)
        got = bb.attn_layer_step(a, 1, W, x, pos=100 + i, theta=THETA)
        q = bb.matvec(bb.GGML_Q4_K, wq, HID, HID, x)
        k = bb.matvec(bb.GGML_Q4_K, wk, HID, KVD, x)
        v = bb.matvec(bb.GGML_Q6_K, wv, HID, KVD, x)
        att = b.attn_step(1, q, k, v, qg, kg, pos=100 + i, theta=THETA)
        np.testing.assert_array_equal(got, bb.matvec(bb.GGML_Q4_K, wo, HID, HID, att))
        # the oracle's composition of the reference arithmetic
        rq = oracle.matvec(oracle.GG_Q4_K, wq, HID, HID, x)
        rk = oracle.matvec(oracle.GG_Q4_K, wk, HID, KVD, x)
        rv = oracle.matvec(oracle.GG_Q6_K, wv, HID, KVD, x)
        np.testing.assert_array_equal(q, rq)
        ratt = ref.attn_step(1, rq, rk, rv, qg, kg, THETA, EPS, H, KVH, D, pos=100 + i)
        want = oracle.matvec(oracle.GG_Q4_K, wo, HID, HID, ratt)
        assert np.abs(got - want).max() <= 5e-3 * max(1.0, np.abs(want).max()), np.abs(got - want).max()
    W.close()


@pytest.mark.parametrize("tensor_cores", [False, True])
def test_layer_batch_against_its_pieces_and_the_oracle(tensor_cores):
    W, (wq, wk, wv, wo, qg, kg) = _layer(seed=7)
    c = bb.Cache(n_layers=1, max_context=512)
    ref = oracle.Cache(1, KVD)
    pos0 = 0
    for t in (40, 70):  # a chunk into an empty cache, then one on top of it
        x = _x(30 + t, (t, HID))
        got = bb.attn_layer_batch(c, 0, W, x, pos0, tensor_cores=tensor_cores, theta=THETA)
        rq = oracle.matmul(oracle.GG_Q4_K, wq, HID, HID, x, t)
        rk = oracle.matmul(oracle.GG_Q4_K, wk, HID, KVD, x, t)
        rv = oracle.matmul(oracle.GG_Q6_K, wv, HID, KVD, x, t)
        ck = ref.k[0] if ref.k[0].shape[0] else None
        cv = ref.v[0] if ref.v[0].shape[0] else None
        ratt, ref.k[0], ref.v[0], _, _ = oracle.attn_batch(rq, rk, rv, pos0, qg, kg, THETA, EPS, H, KVH, D, ck, cv,
                                                           n_threads=oracle.max_threads())
        want = oracle.matmul(oracle.GG_Q4_K, wo, HID, HID, ratt, t)
        err = np.abs(got - want).max() / max(1.0, np.abs(want).max())
        assert err <= (3e-2 if tensor_cores else 5e-3), err
        pos0 += t
    assert c.kv_len() == 110
    if not tensor_cores:  # the fp32 path composes bit for bit
        d = bb.Cache(n_layers=1, max_context=512)
        x = _x(99, (40, HID))
        got = bb.attn_layer_batch(d, 0, W, x, 0, tensor_cores=False, theta=THETA)
        e = bb.Cache(n_layers=1, max_context=512)
        q = bb.matmul(bb.GGML_Q4_K, wq, HID, HID, x, 40)
        k = bb.matmul(bb.GGML_Q4_K, wk, HID, KVD, x, 40)
        v = bb.matmul(bb.GGML_Q6_K, wv, HID, KVD, x, 40)
        att = e.attn_prefill(0, q, k, v, qg, kg, 0, theta=THETA)
        np.testing.assert_array_equal(got, bb.matmul(bb.GGML_Q4_K, wo, HID, HID, att, 40))
    W.close()


def test_whole_operator_step_plans_eager_and_in_a_graph():
    """Whole-operator plans (projections + plan decode + W_o) for two layers against
    attn_layer_step on a copy of the cache, eagerly and replayed from a CUDA graph. The plan's
    decode splits differ from the ordinary step's (last-bit differences in the attention
    output), which W_o's Q8 re-quantization can carry to one quantum."""
    torch = pytest.importorskip("torch")
    W, _ = _layer(seed=11)
    dev = torch.device("cuda", 0)
    a = bb.Cache(n_layers=2, max_context=400)
    for layer in range(2):
        a.append(layer, oracle.normal(40 + layer, (300, KVD)), oracle.normal(50 + layer, (300, KVD)))
    a.pos = 300
    b = a.clone()
    plans = [bb.StepPlan(b, layer, weights=W) for layer in range(2)]
    sx = torch.zeros(HID, device=dev)
    outs = [torch.empty(HID, device=dev) for _ in range(2)]
    graph, cap = torch.cuda.CUDAGraph(), torch.cuda.Stream()
    for i in range(12):
        x = torch.from_numpy(_x(200 + i, HID)).to(dev)
        sx.copy_(x)
        if i < 2:
            for layer in range(2):
                plans[layer].launch_layer(sx, outs[layer], theta=THETA)
        else:
            if i == 2:
                torch.cuda.synchronize()
                with torch.cuda.graph(graph, stream=cap):
                    for layer in range(2):
                        plans[layer].launch_layer(sx, outs[layer], theta=THETA)
            graph.replay()
        for layer in range(2):
            want = bb.attn_layer_step(a, layer, W, x.cpu().numpy(), pos=300 + i, theta=THETA)
            got = outs[layer].cpu().numpy()
            assert np.abs(got - want).max() <= 5e-3 * max(1.0, np.abs(want).max()), (i, layer)
    assert plans[0].steps() == 12
    for p in plans:
        p.finish()
    assert b.kv_len() == a.kv_len() == 312 and b.pos == 312
    np.testing.assert_array_equal(b.read(1)[0], a.read(1)[0])
    W.close()


def test_layer_step_at_a_ragged_shape():
    """hidden 768 (3 blocks per row: the one-token kernel's lanes per row are padded to 4),
    8 query / 2 kv heads, Q6_K on k and W_o: the one call equals its pieces bit for bit."""
    hid, nh, nkv = 768, 8, 2
    wq, wk = random_q4k(nh * D, hid, 61), random_q6k(nkv * D, hid, 62)
    wv, wo = random_q4k(nkv * D, hid, 63), random_q6k(hid, nh * D, 64)
    qg, kg = (1 + 0.02 * oracle.normal(s, D) for s in (65, 66))
    W = bb.AttnWeights((bb.GGML_Q4_K, wq), (bb.GGML_Q6_K, wk), (bb.GGML_Q4_K, wv), (bb.GGML_Q6_K, wo), qg, kg,
                       n_heads=nh, n_kv_heads=nkv, hidden=hid)
    a = bb.Cache(n_layers=1, n_kv_heads=nkv, max_context=256)
    b = a.clone()
    for i in range(4):
        x = _x(300 + i, hid)
        got = bb.attn_layer_step(a, 0, W, x, pos=i, theta=THETA)
        q = bb.matvec(bb.GGML_Q4_K, wq, hid, nh * D, x)
        k = bb.matvec(bb.GGML_Q6_K, wk, hid, nkv * D, x)
        v = bb.matvec(bb.GGML_Q4_K, wv, hid, nkv * D, x)
        att = b.attn_step(0, q, k, v, qg, kg, pos=i, theta=THETA)
        np.testing.assert_array_equal(got, bb.matvec(bb.GGML_Q6_K, wo, nh * D, hid, att))
        np.testing.assert_array_equal(q, oracle.matvec(oracle.GG_Q4_K, wq, hid, nh * D, x))
    W.close()
