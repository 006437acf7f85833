"""The logits head and greedy sampling through the C-ABI against the CPU oracle.

Model::logits_from_hidden (src/model.rs:379-388) is the final RMSNorm followed by the tied
token_embd matvec; Sampler::sample with temperature <= 0 (src/sampler.rs:64-88) is the
presence penalty followed by argmax (:139-149). The matvec is bit-exact against the oracle
for K-quant and F16 weights; the norm's f64 sum of squares is a fixed tree on the GPU, which
equals the reference's sequential f64 sum whenever the partial sums are exact in f64 (as they
are for these inputs), so logits and tokens must match exactly.
"""
import numpy as np
import pytest
import torch

import bebelm_b200 as bb
import oracle
from test_gpu_quant import random_q4k, random_q6k

pytestmark = pytest.mark.gpu


def test_sampler_kats_through_the_c_abi(kats):
    for c in kats["sampler"]:
        logits = np.array(c["logits"], np.float32)
        assert bb.sample_greedy(logits, c["history"], c["repeat_penalty"]) == c["token"], c["src"]
        dl = torch.tensor(c["logits"], dtype=torch.float32, device="cuda")
        tok = bb.sample_greedy(dl, c["history"], c["repeat_penalty"])
        assert int(tok.item()) == c["token"], c["src"]
    logits = np.array([10.0, 4.0, -1.0], np.float32)
    bb.sample_greedy(logits, [0, 0, 2], 2.0)
    assert list(logits) == [5.0, 4.0, -2.0]


def test_argmax_edge_cases_match_the_oracle():
    nan, inf = np.float32("nan"), np.float32("inf")
    cases = [np.array(v, np.float32) for v in ([2, 5, 5, 1], [nan, 1, nan, 3], [-inf, -inf], [nan, nan], [-0.0, 0.0],
                                               [-inf, -3.0], [7.0])]
    rng = np.random.default_rng(5)
    big = rng.standard_normal(65536).astype(np.float32)
    big[[100, 40000, 65535]] = 9.5  # ties far apart: the first one
    big[rng.integers(0, 65536, 300)] = nan
    cases.append(big)
    for v in cases:
        want = oracle.argmax(v)
        assert bb.sample_greedy(v.copy()) == want
        assert int(bb.sample_greedy(torch.from_numpy(v.copy()).cuda()).item()) == want
    # the penalty on the device: a large history with repeats, logits rewritten in place
    logits = rng.standard_normal(50000).astype(np.float32) * 4
    hist = rng.integers(0, 50000, 3000).astype(np.uint32)
    want_l = logits.copy()
    want = oracle.sample_greedy(want_l, hist, 1.3)
    dl = torch.from_numpy(logits.copy()).cuda()
    got = bb.sample_greedy(dl, torch.from_numpy(hist.astype(np.int32)).cuda(), 1.3)
    assert int(got.item()) == want
    np.testing.assert_array_equal(dl.cpu().numpy(), want_l)
    hl = logits.copy()
    assert bb.sample_greedy(hl, hist, 1.3) == want
    np.testing.assert_array_equal(hl, want_l)


@pytest.mark.parametrize("dtype,gen,vocab", [(bb.GGML_Q6_K, random_q6k, 3000), (bb.GGML_Q4_K, random_q4k, 3000),
                                             (bb.GGML_F16, None, 3000), (bb.GGML_Q6_K, random_q6k, 20000),
                                             (bb.GGML_Q4_K, random_q4k, 12345), (bb.GGML_Q6_K, random_q6k, 128000)])
def test_logits_head_matches_the_oracle(dtype, gen, vocab):
    """Small vocabularies take the lane kernel; from 8192 rows K-quants stream through shared
    memory (ragged last chunk at 12345 rows; at the model's 128000 rows each CTA streams ~27
    chunks, alternating between its two warp groups)."""
    hidden = 2048
    if gen is None:
        w = (np.random.default_rng(3).standard_normal((vocab, hidden)) * 0.02).astype(np.float16).view(np.uint8)
        w = w.reshape(-1)
    else:
        w = gen(vocab, hidden, seed=vocab)
    gain = (1 + 0.1 * oracle.normal(8, hidden)).astype(np.float32)
    head = bb.Head(dtype, w, hidden, vocab, gain)
    for seed in range(3):
        h = oracle.normal(30 + seed, hidden) * 3
        want = oracle.logits_head(dtype, w, hidden, vocab, gain, h)
        lg, tok = head.logits(h)
        np.testing.assert_array_equal(lg, want)
        assert tok == oracle.argmax(want)
        # device: everything stays on the GPU (token as a device int32)
        dlg, dtok = head.logits(torch.from_numpy(h).cuda())
        np.testing.assert_array_equal(dlg.cpu().numpy(), want)
        assert int(dtok.item()) == tok
        _, only_tok = head.logits(torch.from_numpy(h).cuda(), logits=False)
        assert int(only_tok.item()) == tok
    head.close()


def test_greedy_head_in_a_cuda_graph():
    """The head's device call captured in a CUDA graph: replays pick the argmax of the current
    hidden state (an on-device greedy loop needs no host round trip)."""
    hidden, vocab = 2048, 4096
    w = random_q6k(vocab, hidden, seed=1)
    gain = np.ones(hidden, np.float32)
    head = bb.Head(bb.GGML_Q6_K, w, hidden, vocab, gain)
    hs = torch.zeros(hidden, device="cuda")
    tok = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.Stream()
    g = torch.cuda.CUDAGraph()
    head.logits(hs.normal_(), stream=stream)  # warm-up outside the capture
    torch.cuda.synchronize()
    with torch.cuda.graph(g, stream=stream):
        bb.load_library().bebelm_head_logits(head._h, hs.data_ptr(), 1e-5, None, tok.data_ptr(), bb.MEM_DEVICE,
                                             stream.cuda_stream)
    for seed in range(4):
        h = oracle.normal(70 + seed, hidden)
        hs.copy_(torch.from_numpy(h))
        g.replay()
        torch.cuda.synchronize()
        assert int(tok.item()) == oracle.argmax(oracle.logits_head(bb.GGML_Q6_K, w, hidden, vocab, gain, h))
    head.close()
