"""Quantized products through the C-ABI against the CPU oracle (src/kernels/matmul.rs, dequant.rs).

K-quant weights (Q4_K, Q6_K) go through the reference's Q8-activation integer dot, which is
exact in its integer part and written in the reference's f32 order: the GPU must equal the
oracle bit for bit. F32/F16 weights follow the reference's `dot` structure, in the oracle's
(unpinned) final-reduction order: also bit for bit against the oracle.
"""
import numpy as np
import pytest

import bebelm_b200 as bb
import oracle
from test_oracle_kats import _patched, q4k_test_block, q6k_test_block

pytestmark = pytest.mark.gpu


def random_q4k(rows, n_in, seed):
    rng = np.random.default_rng(seed)
    w = rng.integers(0, 256, size=(rows, n_in // 256, 144), dtype=np.uint8)
    d = (rng.standard_normal((rows, n_in // 256)) * 0.01).astype(np.float16).view(np.uint8).reshape(rows, -1, 2)
    dm = (np.abs(rng.standard_normal((rows, n_in // 256))) * 0.005).astype(np.float16).view(np.uint8).reshape(rows, -1, 2)
    w[:, :, 0:2], w[:, :, 2:4] = d, dm
    return w.reshape(-1)


def random_q6k(rows, n_in, seed):
    rng = np.random.default_rng(seed)
    w = rng.integers(0, 256, size=(rows, n_in // 256, 210), dtype=np.uint8)
    d = (rng.standard_normal((rows, n_in // 256)) * 0.002).astype(np.float16).view(np.uint8).reshape(rows, -1, 2)
    w[:, :, 208:210] = d
    return w.reshape(-1)


def test_kats_through_the_c_abi(kats):
    q = kats["quant"]
    bits = np.array([b for b, _ in q["f16"]["exact"]] + q["f16"]["nan"], np.uint16)
    got = bb.dequantize(bb.GGML_F16, bits.view(np.uint8), bits.size)
    for (b, val), g in zip(q["f16"]["exact"], got):
        assert g == float(val) and np.signbit(g) == np.signbit(float(val)), b
    assert np.isnan(got[-1])
    for name, dtype in (("q4k_block", bb.GGML_Q4_K), ("q6k_block", bb.GGML_Q6_K)):
        out = bb.dequantize(dtype, _patched(q[name]), 256)
        assert all(out[int(i)] == v for i, v in q[name]["out"].items()), name
    two = bb.dequantize(bb.GGML_Q4_K, _patched(q["dispatch_two_q4k"], 2), 512)
    assert two[0] == 7.0 and two[256] == 7.0
    c = q["matvec_f32_small"]
    w = np.array(c["w"], np.float32).view(np.uint8)
    for x, want in c["cases"]:
        assert list(bb.matvec(bb.GGML_F32, w, 2, 3, np.array(x, np.float32))) == want
    c = q["matvec_f16_small"]
    assert list(bb.matvec(bb.GGML_F16, np.array(c["bits"], np.uint16).view(np.uint8), 2, 3,
                          np.array(c["x"], np.float32))) == c["out"]
    x = np.zeros(256, np.float32)
    x[0] = 1.0
    assert bb.matvec(bb.GGML_Q4_K, _patched(q["matvec_q4k_single_row"]), 256, 1, x)[0] == 7.0
    for blk, x in (q4k_test_block(), ):
        assert bb.matvec(bb.GGML_Q4_K, blk, 256, 1, x)[0] == oracle.matvec(oracle.GG_Q4_K, blk, 256, 1, x)[0]
    blk, x = q6k_test_block()
    assert bb.matvec(bb.GGML_Q6_K, blk, 256, 1, x)[0] == oracle.matvec(oracle.GG_Q6_K, blk, 256, 1, x)[0]


@pytest.mark.parametrize("dtype,gen,n_out", [(bb.GGML_Q4_K, random_q4k, 2048), (bb.GGML_Q4_K, random_q4k, 512),
                                             (bb.GGML_Q6_K, random_q6k, 512), (bb.GGML_Q6_K, random_q6k, 2048)])
def test_projection_shapes_bit_exact(dtype, gen, n_out):
    """The q/o (2048 x 2048) and k/v (512 x 2048) projection shapes, seeded activations."""
    n_in = 2048
    w = gen(n_out, n_in, seed=n_out + dtype)
    x = oracle.normal(40 + dtype, n_in)
    np.testing.assert_array_equal(bb.matvec(dtype, w, n_in, n_out, x), oracle.matvec(dtype, w, n_in, n_out, x))
    # several tokens at once (the prefill projection): matvec per token, bit for bit
    xs = oracle.normal(50 + dtype, (5, n_in))
    np.testing.assert_array_equal(bb.matmul(dtype, w, n_in, n_out, xs, 5), oracle.matmul(dtype, w, n_in, n_out, xs, 5))
    np.testing.assert_array_equal(bb.dequantize(dtype, w, n_out * n_in), oracle.dequantize(dtype, w, n_out * n_in))


@pytest.mark.parametrize("dtype", [bb.GGML_F32, bb.GGML_F16])
def test_float_weights_match_the_oracle(dtype):
    rng = np.random.default_rng(dtype)
    for n_in, n_out in ((520, 300), (2048, 64), (7, 5), (40, 128)):
        wf = rng.standard_normal((n_out, n_in)).astype(np.float32)
        w = (wf if dtype == bb.GGML_F32 else wf.astype(np.float16)).view(np.uint8).reshape(-1)
        x = rng.standard_normal(n_in).astype(np.float32)
        np.testing.assert_array_equal(bb.matvec(dtype, w, n_in, n_out, x), oracle.matvec(dtype, w, n_in, n_out, x))


def test_edge_activations_and_device_buffers():
    torch = pytest.importorskip("torch")
    w = random_q4k(64, 512, seed=9)
    for x in (np.zeros(512, np.float32),                       # max|x| = 0: every quant 0
              np.full(512, 3.0e30, np.float32),                # large magnitudes
              np.where(np.arange(512) % 2, 1.0, -1.0).astype(np.float32) * 0.5):  # exact .5 ties
        np.testing.assert_array_equal(bb.matvec(bb.GGML_Q4_K, w, 512, 64, x), oracle.matvec(oracle.GG_Q4_K, w, 512, 64, x))
    # device buffers: the same bits
    x = oracle.normal(77, 512)
    dw = torch.from_numpy(w).cuda()
    dx = torch.from_numpy(x).cuda()
    got = bb.matvec(bb.GGML_Q4_K, dw, 512, 64, dx).cpu().numpy().reshape(-1)
    np.testing.assert_array_equal(got, oracle.matvec(oracle.GG_Q4_K, w, 512, 64, x))
    with pytest.raises(bb.BebelmError):
        bb.matvec(bb.GGML_Q4_K, w, 500, 64, np.zeros(500, np.float32))  # not a multiple of 256
    with pytest.raises(bb.BebelmError):
        bb.matvec(2, w, 512, 64, x)  # Q4_0: not supported


@pytest.mark.parametrize("dtype,gen", [(bb.GGML_Q4_K, random_q4k), (bb.GGML_Q6_K, random_q6k)])
@pytest.mark.parametrize("n_out,n_in,t", [(100, 512, 70), (512, 2048, 64), (130, 256, 33)])
def test_tiled_matmul_bit_exact(dtype, gen, n_out, n_in, t):
    """Many tokens take the 64 x 64 tiled kernel: ragged rows and tokens, same bits as matvec."""
    w = gen(n_out, n_in, seed=n_out * 7 + t)
    xs = oracle.normal(90 + t, (t, n_in))
    xs[3] = 0.0  # a token whose quants are all zero
    np.testing.assert_array_equal(bb.matmul(dtype, w, n_in, n_out, xs, t), oracle.matmul(dtype, w, n_in, n_out, xs, t))


@pytest.mark.parametrize("dtype,gen,n_out,n_in,t", [
    (bb.GGML_Q4_K, random_q4k, 300, 1024, 200), (bb.GGML_Q4_K, random_q4k, 2048, 2048, 128),
    (bb.GGML_Q4_K, random_q4k, 128, 256, 64),
    (bb.GGML_Q6_K, random_q6k, 512, 2048, 130), (bb.GGML_Q6_K, random_q6k, 200, 4096, 64),
    (bb.GGML_Q6_K, random_q6k, 96, 1024, 70)])  # n_in 1024: Q6_K rows not 16-byte multiples -> dp4a
def test_kquant_tensor_core_matmul_bit_exact(dtype, gen, n_out, n_in, t):
    """From 64 tokens on, K-quants take the tensor-core kernel (tcgen05 kind::i8, exact integer
    sub-block dots): ragged row and token tiles, a zero token and a saturated token, same bits."""
    w = gen(n_out, n_in, seed=n_out + t)
    xs = oracle.normal(120 + t, (t, n_in))
    xs[5] = 0.0
    xs[t - 1] = np.where(np.arange(n_in) % 3, 1e3, -1e3)  # every quant at +-127
    xs[t - 2] = 1e3   # sub-block sums at +4064: the Q4_K min term's split 64 * 63 + 32
    xs[t - 3] = -1e3  # and at -4064: 64 * (-64) + 32
    np.testing.assert_array_equal(bb.matmul(dtype, w, n_in, n_out, xs, t),
                                  oracle.matmul(dtype, w, n_in, n_out, xs, t))
