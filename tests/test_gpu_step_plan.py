"""Step plans (device-driven decode steps) against the ordinary fused step, through the C-ABI.

The ordinary equivalent of plan step n with window W is: evict the oldest position when the
layer holds W already, then attn_step at position pos + n (src/model.rs:440-451 with the
sliding window of src/agent.rs:466-476). The appended K/V must be bit-identical (same
arithmetic); the attention output may differ in the last bits because the plan's split
boundaries are fixed for the largest window.
"""
import numpy as np
import pytest
import torch

import bebelm_b200 as bb
import oracle

pytestmark = pytest.mark.gpu

H, KVH, D = 32, 8, 64
HID, KVD = H * D, KVH * D
THETA = 1e6
ATOL = 1e-5  # split-boundary rounding only


def _setup(t0=700, max_context=1024, seed=3):
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(seed)
    a = bb.Cache(n_layers=2, max_context=max_context)
    for layer in range(2):
        a.append(layer, torch.randn((t0, KVD), generator=g, device=dev), torch.randn((t0, KVD), generator=g, device=dev))
    a.pos = t0
    qg = 1 + 0.02 * torch.randn(D, generator=g, device=dev)
    kg = 1 + 0.02 * torch.randn(D, generator=g, device=dev)
    return a, qg, kg, g, dev


def test_plan_steps_match_ordinary_steps_while_the_window_slides():
    a, qg, kg, g, dev = _setup()
    b = a.clone()
    W, n_steps, p0 = 720, 48, a.pos
    plans = [b.step_plan(layer, window=W) for layer in range(2)]
    with pytest.raises(bb.BebelmError):
        b.kv_len()  # the device owns the window while plans are open
    out = torch.empty(HID, device=dev)
    for i in range(n_steps):
        q, k, v = (torch.randn(n, generator=g, device=dev) for n in (HID, KVD, KVD))
        if a.kv_len() >= W:
            a.evict_front(1)
        for layer in range(2):
            want = a.attn_step(layer, q, k, v, qg, kg, pos=p0 + i, theta=THETA)
            got = plans[layer].launch(q, k, v, qg, kg, out, theta=THETA)
            np.testing.assert_allclose(got.cpu().numpy(), want.cpu().numpy(), atol=ATOL, rtol=0)
    assert plans[0].steps() == n_steps
    for p in plans:
        p.finish()
    assert b.kv_len() == a.kv_len() == W
    assert b.pos == p0 + n_steps
    for layer in range(2):
        assert b.layer_len(layer) == a.layer_len(layer)
        ka, va = a.read(layer)
        kb, vb = b.read(layer)
        np.testing.assert_array_equal(kb, ka)
        np.testing.assert_array_equal(vb, va)
    # ordinary calls work again and agree
    q, k, v = (torch.randn(n, generator=g, device=dev) for n in (HID, KVD, KVD))
    a.evict_front(1)
    b.evict_front(1)
    np.testing.assert_allclose(b.attn_step(0, q, k, v, qg, kg, pos=p0 + n_steps, theta=THETA).cpu().numpy(),
                               a.attn_step(0, q, k, v, qg, kg, pos=p0 + n_steps, theta=THETA).cpu().numpy(),
                               atol=ATOL, rtol=0)


def test_plan_steps_captured_in_a_cuda_graph():
    a, qg, kg, g, dev = _setup(t0=1000, max_context=1024, seed=5)
    b = a.clone()
    W, p0 = 1024, a.pos
    plans = [b.step_plan(layer, window=W) for layer in range(2)]
    sq, sk, sv = (torch.zeros(n, device=dev) for n in (HID, KVD, KVD))
    outs = [torch.empty(HID, device=dev) for _ in range(2)]
    # one eager step first (plan step 0), then capture one step of both layers
    inputs = [tuple(torch.randn(n, generator=g, device=dev) for n in (HID, KVD, KVD)) for _ in range(40)]
    graph = torch.cuda.CUDAGraph()
    stream = torch.cuda.Stream()
    torch.cuda.synchronize()
    for i, (q, k, v) in enumerate(inputs):
        sq.copy_(q), sk.copy_(k), sv.copy_(v)
        if i == 0:
            for layer in range(2):
                plans[layer].launch(sq, sk, sv, qg, kg, outs[layer], theta=THETA)
        elif i == 1:
            with torch.cuda.graph(graph, stream=stream):
                for layer in range(2):
                    plans[layer].launch(sq, sk, sv, qg, kg, outs[layer], theta=THETA)
            graph.replay()  # capture does not run the kernels
        else:
            graph.replay()
        got = [o.cpu().numpy() for o in outs]
        if a.kv_len() >= W:
            a.evict_front(1)
        for layer in range(2):
            want = a.attn_step(layer, q, k, v, qg, kg, pos=p0 + i, theta=THETA).cpu().numpy()
            np.testing.assert_allclose(got[layer], want, atol=ATOL, rtol=0)
    assert plans[1].steps() == len(inputs)
    for p in plans:
        p.finish()
    assert b.kv_len() == a.kv_len() and b.pos == p0 + len(inputs)
    np.testing.assert_array_equal(b.read(1)[0], a.read(1)[0])


def test_plan_against_the_oracle_on_an_empty_layer_window():
    """A plan started on a short window: every step against the CPU oracle (1e-3)."""
    dev = torch.device("cuda", 0)
    c = bb.Cache(n_layers=1, max_context=256)
    ref = oracle.Cache(1, KVD)
    qg, kg = (1 + 0.02 * oracle.normal(s, D) for s in (61, 62))
    plan = c.step_plan(0, window=100)
    out = torch.empty(HID, device=dev)
    dqg, dkg = torch.from_numpy(qg).to(dev), torch.from_numpy(kg).to(dev)
    for i in range(130):
        q, k, v = oracle.normal(300 + i, HID), oracle.normal(600 + i, KVD), oracle.normal(900 + i, KVD)
        got = plan.launch(*(torch.from_numpy(x).to(dev) for x in (q, k, v)), dqg, dkg, out, theta=THETA)
        if ref.kv_len() >= 100:
            ref.evict_front(1)
        want = ref.attn_step(0, q, k, v, qg, kg, THETA, 1e-5, H, KVH, D, pos=i)
        np.testing.assert_allclose(got.cpu().numpy(), want, atol=1e-3, rtol=0)
    plan.finish()
    assert c.kv_len() == 100 and c.pos == 130
