"""Benchmark of the GQA decode hot path at a 32k sliding window.

One step = one decode step of one attention layer on a full 32768-position
window (32 q heads / 8 kv heads, d=64, fp32 KV): q/k norm + RoPE at the next
position, KV append, split-K attention over the 32769 cached positions, and
eviction of the oldest position (the max_context sliding window). The metric
is the algorithmic KV-read bandwidth: 2 (K and V) x positions x 512 x 4 bytes
per step, each byte counted once (the reference re-reads it per query head).

With --gpus N (torchrun, one process per GPU) every rank runs its own sequence
(per-sequence sharding, no collective): "scaling": "weak".

--impl reference times the reference's CPU arithmetic (the C restatement in
oracle/, since the Rust crate cannot be built in this image) on the host cores
for the same step, on rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CTX = 32768
H, KVH, D = 32, 8, 64
HID, KVD = H * D, KVH * D
THETA, EPS = 1e6, 1e-5
METRIC = "decode-attn KV-read GB/s @32k ctx (1 layer, 32q/8kv, d=64, fp32 KV)"


def workload_config(world: int) -> dict:
    """The workload, identical in both arms' JSON lines."""
    return {"workload": "config3: 1 seq per GPU, 32768-position window, append+evict per step",
            "n_ctx": CTX, "heads": "32q/8kv", "head_dim": D, "theta": THETA, "kv_dtype": "f32",
            "parallelism": f"per-sequence x{world}",
            "l2": "no flush: the 134 MB window exceeds the 126 MB L2"}


def bytes_per_step(n_ctx: int) -> int:
    return 2 * n_ctx * KVD * 4


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            j = json.load(f)
        return float(j["hbm_gbs"]), float(j["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


class Clocks:
    """nvidia-smi sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, dev: int):
        self.dev = dev
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-i", str(self.dev),
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out = ""
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_setup(backend):
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        dist.init_process_group(backend)
    return world, rank, local


def max_over_ranks(x: float, world: int, device) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


# ---------------------------------------------------------------- CPU side --
def cpu_decode_sample(threads: int, budget_s: float, steps_max: int, seed: int = 7):
    """The reference's decode step on the host: norm/RoPE, append into a Vec-like buffer,
    attention_decode over the window, evict_front(1) by a memmove of the remaining rows
    (src/cache.rs:44-45 drains the front). Returns (seconds per step, steps done)."""
    import numpy as np

    import oracle
    rng = np.random.default_rng(seed)
    ck = rng.standard_normal((CTX + 1, KVD), dtype=np.float32)
    cv = rng.standard_normal((CTX + 1, KVD), dtype=np.float32)
    qg = (1 + 0.02 * rng.standard_normal(D)).astype(np.float32)
    kg = (1 + 0.02 * rng.standard_normal(D)).astype(np.float32)
    done, t_total = 0, 0.0
    while done < steps_max and (t_total < budget_s or done == 0):
        q = rng.standard_normal(HID, dtype=np.float32)
        k = rng.standard_normal(KVD, dtype=np.float32)
        v = rng.standard_normal(KVD, dtype=np.float32)
        t0 = time.perf_counter()
        qn = oracle.norm_rope_heads(q, H, D, qg, CTX + done, THETA, EPS)
        kn = oracle.norm_rope_heads(k, KVH, D, kg, CTX + done, THETA, EPS)
        ck[CTX] = kn
        cv[CTX] = v
        oracle.attention_decode(qn, ck, cv, CTX + 1, H, KVH, D, n_threads=threads)
        ck[:CTX] = ck[1:]
        cv[:CTX] = cv[1:]
        t_total += time.perf_counter() - t0
        done += 1
    return t_total / done, done


def run_reference(args):
    world, rank, local = dist_setup("gloo")
    if rank != 0:
        return 0
    import oracle
    threads = oracle.max_threads()
    # bounded: warm-up steps untimed, then as many of the K steps as fit ~120 s
    cpu_decode_sample(threads, 0.0, max(1, min(args.warmup, 2)))
    sec, done = cpu_decode_sample(threads, 120.0, args.steps)
    value = bytes_per_step(CTX + 1) / sec / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(sec * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0,1))",
        "config": workload_config(world),
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"{done} of {args.steps} decode steps at 32768 positions (oracle C restatement of "
                                   f"src/kernels/attention.rs, heads over {threads} threads)"},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "tok_per_s": round(1.0 / sec, 3),
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------- GPU side --
def run_ours(args):
    import numpy as np
    import torch

    world, rank, local = dist_setup("nccl")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    import bebelm_b200 as bb
    bb.load_library()

    g = torch.Generator(device=dev)
    g.manual_seed(1234 + rank)
    stream = torch.cuda.current_stream()
    cache = bb.Cache(n_layers=1, max_context=CTX, device=local)
    chunk = 4096
    for c0 in range(0, CTX, chunk):
        kk = torch.randn((chunk, KVD), generator=g, device=dev)
        vv = torch.randn((chunk, KVD), generator=g, device=dev)
        cache.append(0, kk, vv)
    n_steps = args.warmup + args.steps
    Q = torch.randn((n_steps, HID), generator=g, device=dev)
    K = torch.randn((n_steps, KVD), generator=g, device=dev)
    V = torch.randn((n_steps, KVD), generator=g, device=dev)
    qg = 1 + 0.02 * torch.randn(D, generator=g, device=dev)
    kg = 1 + 0.02 * torch.randn(D, generator=g, device=dev)
    OUT = torch.empty((n_steps, HID), device=dev)
    pos = [CTX]

    # the C-ABI called as a Rust caller would (device pointers computed once, no per-call
    # wrapper work), so that the host's launch rate does not cap the device-timed step
    lib = bb.load_library()
    sp = stream.cuda_stream
    qp0, kp0, vp0, op0 = Q.data_ptr(), K.data_ptr(), V.data_ptr(), OUT.data_ptr()
    qgp, kgp = qg.data_ptr(), kg.data_ptr()

    def step(i):
        rc = lib.bebelm_attn_step(cache._h, 0, H, qp0 + 4 * HID * i, kp0 + 4 * KVD * i, vp0 + 4 * KVD * i, qgp, kgp,
                                  THETA, EPS, pos[0], op0 + 4 * HID * i, bb.MEM_DEVICE, sp)
        if rc == 0:
            rc = lib.bebelm_kv_evict_front(cache._h, 1)
        if rc != 0:
            raise bb.BebelmError(rc, bb.last_error())
        pos[0] += 1

    for i in range(args.warmup):
        step(i)
    clocks = Clocks(local)
    barrier(world)
    torch.cuda.synchronize()
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.warmup, n_steps):
        step(i)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    clk = clocks.stop()
    ms = max_over_ranks(e0.elapsed_time(e1), world, dev)
    assert torch.isfinite(OUT).all().item()
    total_bytes = bytes_per_step(CTX + 1) * args.steps * world
    value = total_bytes / (ms * 1e-3) / 1e9

    # -- dominant kernel alone: split-K decode over the 32768 window (events per launch)
    qn = Q[0].clone()
    bb.norm_rope_heads(qn, H, D, qg, CTX, THETA, EPS, stream=stream)
    dout = torch.empty(HID, device=dev)
    for _ in range(5):
        cache.decode(0, qn, out=dout, stream=stream)
    reps = 50
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
    for a, b in evs:
        a.record(stream)
        cache.decode(0, qn, out=dout, stream=stream)
        b.record(stream)
    torch.cuda.synchronize()
    kern_ms = statistics.mean(a.elapsed_time(b) for a, b in evs)
    hbm_peak, bf16_peak, peak_kind = peaks()
    # the timed region launches decode_kernel alone, once per step: its average duration
    # there (PDL-chained) is the timed time per step
    achieved = bytes_per_step(CTX + 1) / (ms / args.steps * 1e-3) / 1e9
    isolated = bytes_per_step(CTX) / (kern_ms * 1e-3) / 1e9
    traffic, traffic_src = load_profile_traffic()

    # -- end to end through the C-ABI with host buffers: the call a Rust caller makes per step
    #    (bebelm_attn_step with mem = HOST: inputs copied in and the output back inside the
    #    call, which returns once the output is in the caller's memory) plus evict_front
    e2e_steps = min(args.steps, 128)
    rs = np.random.default_rng(99 + rank)
    hq = rs.standard_normal((e2e_steps, HID), dtype=np.float32)
    hk = rs.standard_normal((e2e_steps, KVD), dtype=np.float32)
    hv = rs.standard_normal((e2e_steps, KVD), dtype=np.float32)
    hqg, hkg = qg.cpu().numpy(), kg.cpu().numpy()
    hout = np.zeros(HID, np.float32)
    lib = bb.load_library()
    qp, kp, vp, gqp, gkp, op = (x.ctypes.data for x in (hq, hk, hv, hqg, hkg, hout))

    def e2e_step(i):
        rc = lib.bebelm_attn_step(cache._h, 0, H, qp + 4 * HID * i, kp + 4 * KVD * i, vp + 4 * KVD * i, gqp, gkp,
                                  THETA, 1e-5, pos[0], op, bb.MEM_HOST, None)
        if rc == 0:
            rc = lib.bebelm_kv_evict_front(cache._h, 1)
        if rc != 0:
            raise bb.BebelmError(rc, bb.last_error())
        pos[0] += 1

    e2e_step(0)
    barrier(world)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        e2e_step(i)
    e2e_s = max_over_ranks(time.perf_counter() - t0, world, dev)
    e2e_value = bytes_per_step(CTX + 1) * e2e_steps * world / e2e_s / 1e9

    # -- secondary: config 2 causal prefill (2048 tokens, bf16 inputs)
    prefill = None
    if rank == 0 and not args.no_prefill:
        prefill = {"attn_layer": bench_attn_layer(bb, torch, dev, stream),
                   "config2_2048": bench_prefill(bb, torch, dev, stream, bf16_peak, peak_kind, 2048, 6),
                   "config5_8192_one_layer": bench_prefill(bb, torch, dev, stream, bf16_peak, peak_kind, 8192, 2),
                   "f32_host_inputs": bench_prefill_f32_host(bb, torch, bf16_peak, peak_kind)}

    head = bench_logits_head(bb, torch, dev, stream, hbm_peak, peak_kind) if rank == 0 and not args.no_prefill else None
    c3bf = bench_config3_narrow(bb, torch, dev, stream, world, args.steps, bb.BF16)
    c3f8 = bench_config3_narrow(bb, torch, dev, stream, world, args.steps, bb.FP8)
    cfg4 = None if args.no_cfg4 else bench_config4(bb, torch, dev, stream, world, rank)
    hbm_peak_, bf16_peak_, _ = peaks()
    cfg5 = None if args.no_cfg5 else bench_config5(bb, torch, dev, stream, world, rank, bf16_peak_)

    cpu = cpu1 = None
    if rank == 0 and world == 1 and not args.no_cpu:
        import oracle
        threads = oracle.max_threads()
        sec, done = cpu_decode_sample(threads, 15.0, 64)
        cpu = {"value": round(bytes_per_step(CTX + 1) / sec / 1e9, 3), "unit": "GB/s", "cores": threads,
               "kind": "port",
               "sample": f"{done} decode steps at 32768 positions on {threads} threads (C restatement of the "
                         f"reference arithmetic, heads spread over threads by the harness; the reference itself "
                         f"runs attention on 1 core)"}
        sec1, done1 = cpu_decode_sample(1, 10.0, 16)
        cpu1 = {"value": round(bytes_per_step(CTX + 1) / sec1 / 1e9, 4), "unit": "GB/s", "cores": 1, "kind": "port",
                "sample": f"{done1} decode steps at 32768 positions on 1 thread (serial, as the reference's "
                          f"attention_decode runs)"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0,1))",
            "config": workload_config(world),
            "tok_per_s": round(args.steps * world / (ms * 1e-3), 1),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                         "frac": round(achieved / hbm_peak, 4), "peak_kind": peak_kind,
                         "kernel": "decode_kernel<4> (fused step: norm/RoPE/append + split-K + combine)",
                         "kernel_us": round(ms / args.steps * 1e3, 2),
                         "isolated_launch": {"us": round(kern_ms * 1e3, 2), "gbs": round(isolated, 1),
                                             "note": "one launch between events, no PDL overlap"},
                         "traffic": traffic, "traffic_source": traffic_src},
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": 4 * (HID + 2 * KVD + 2 * D),
                    "d2h_bytes_per_step": 4 * HID, "steps": e2e_steps},
            "gpu_launches": args.steps,
            "clocks": clk,
            "cpu_baseline": cpu,
            "cpu_baseline_1core": cpu1,
            "prefill": prefill,
            "config3_bf16_kv": c3bf,
            "config3_fp8_kv": c3f8,
            "logits_head": head,
            "config4": cfg4,
            "config5": cfg5,
        }
        print(json.dumps(line), flush=True)
    barrier(world)
    return 0


def load_profile_traffic():
    """DRAM bytes per decode launch and where they come from: the committed ncu summary of the
    decode kernel (an ncu capture cannot run inside this timed process). The summary names the
    commit of the kernel source it captured; the line carries that label so a stale figure shows."""
    p = os.path.join(ROOT, "profiles", "decode_kernel_config3.md")
    val, src = None, None
    try:
        with open(p) as f:
            for line in f:
                if line.startswith("| dram_bytes_per_launch |"):
                    val = int(line.split("|")[2])
                elif line.startswith("| kernel_source_commit |"):
                    src = line.split("|")[2].strip()
    except Exception:
        pass
    return val, f"ncu capture in profiles/decode_kernel_config3.md (decode kernel source of commit {src})"


def bench_prefill(bb, torch, dev, stream, bf16_peak, peak_kind, T=2048, reps=6):
    """Causal prefill of T bf16 tokens into `reps` empty caches, enqueued back to back (each call:
    norm + RoPE + append into the paged cache, then the tensor-core attention)."""
    g = torch.Generator(device=dev)
    g.manual_seed(77)
    q = torch.randn((T, HID), generator=g, device=dev).to(torch.bfloat16)
    k = torch.randn((T, 8 * D), generator=g, device=dev).to(torch.bfloat16)
    v = torch.randn((T, 8 * D), generator=g, device=dev).to(torch.bfloat16)
    qg = 1 + 0.02 * torch.randn(D, generator=g, device=dev)
    kg = 1 + 0.02 * torch.randn(D, generator=g, device=dev)
    out = torch.empty((T, HID), device=dev)
    caches = [bb.Cache(n_layers=1, max_context=T) for _ in range(reps)]
    times = []
    for it in range(4):
        for c in caches:
            c.clear()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for c in caches:
            c.attn_prefill(0, q, k, v, qg, kg, 0, theta=THETA, out=out, stream=stream)
        b.record(stream)
        torch.cuda.synchronize()
        if it >= 1:
            times.append(a.elapsed_time(b) / reps)
    for c in caches:
        c.close()
    ms = statistics.mean(times)
    flops = 4096.0 * T * (T + 1)
    tf = flops / (ms * 1e-3) / 1e12
    return {"workload": f"causal prefill of {T} bf16 tokens into an empty cache (norm+RoPE+append+attention), "
                        f"{reps} caches back to back",
            "ms": round(ms, 4), "value": round(tf, 3), "unit": "TFLOP/s",
            "roofline": {"bound": "tensor", "achieved": round(tf, 3), "peak": bf16_peak, "unit": "TFLOP/s",
                         "frac": round(tf / bf16_peak, 4), "peak_kind": peak_kind}}


def bench_prefill_f32_host(bb, torch, bf16_peak, peak_kind):
    """The drop-in prefill a Rust attn_batch makes (src/model.rs:232-254): fp32 q/k/v in host
    memory through bebelm_attn_prefill with mem = HOST, output back in host memory, the copies
    inside the timed region. BEBELM_F32_TENSOR (tensor cores) at 2048 and 8192 tokens, and the
    reference-arithmetic fp32 path (one causal split-K decode per token) at 2048."""
    import numpy as np
    rng = np.random.default_rng(78)
    out = {}
    for T, tc in ((2048, True), (8192, True), (2048, False)):
        q = rng.standard_normal((T, HID), dtype=np.float32)
        k = rng.standard_normal((T, KVD), dtype=np.float32)
        v = rng.standard_normal((T, KVD), dtype=np.float32)
        qg = (1 + 0.02 * rng.standard_normal(D)).astype(np.float32)
        kg = (1 + 0.02 * rng.standard_normal(D)).astype(np.float32)
        c = bb.Cache(n_layers=1, max_context=T)
        o = np.ones((T, HID), np.float32)  # the caller's output buffer, allocated once (as the model's scratch)
        times = []
        for it in range(3):
            c.clear()
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            c.attn_prefill(0, q, k, v, qg, kg, 0, theta=THETA, tensor_cores=tc, out=o)  # returns once o holds it
            times.append(time.perf_counter() - t0)
        c.close()
        ms = statistics.median(times[1:]) * 1e3
        tf = 4096.0 * T * (T + 1) / (ms * 1e-3) / 1e12
        name = f"{'tensor_cores' if tc else 'fp32_reference_arithmetic'}_{T}"
        out[name] = {"ms": round(ms, 3), "tflops": round(tf, 2), "frac_of_bf16_peak": round(tf / bf16_peak, 4),
                     "h2d_bytes": int(4 * (q.size + k.size + v.size + 2 * D)), "d2h_bytes": int(4 * T * HID)}
    out["how"] = "host fp32 buffers through the C-ABI, wall clock per call (copies in and out included)"
    return out


def bench_attn_layer(bb, torch, dev, stream, T=2048, steps=64):
    """The whole attention operator of a layer (src/model.rs attn_batch / attn_step) on
    device-resident GGML weights (synthetic Q4_K q/k/o and Q6_K v, the usual Q4_K_M mix): a
    T-token chunk into an empty cache (projections over T tokens, tensor-core prefill, output
    projection), then `steps` one-token steps on that window."""
    import numpy as np
    rng = np.random.default_rng(5)

    def qk(rows, n_in, six=False):
        bb_ = 210 if six else 144
        w = rng.integers(0, 256, size=(rows, n_in // 256, bb_), dtype=np.uint8)
        d = (rng.standard_normal((rows, n_in // 256)) * (0.002 if six else 0.01)).astype(np.float16)
        w[:, :, (208 if six else 0):(210 if six else 2)] = d.view(np.uint8).reshape(rows, -1, 2)
        if not six:
            w[:, :, 2:4] = (np.abs(rng.standard_normal((rows, n_in // 256))) * 0.005).astype(
                np.float16).view(np.uint8).reshape(rows, -1, 2)
        return w.reshape(-1)

    qg = (1 + 0.02 * rng.standard_normal(D)).astype(np.float32)
    kg = (1 + 0.02 * rng.standard_normal(D)).astype(np.float32)
    W = bb.AttnWeights((bb.GGML_Q4_K, qk(HID, HID)), (bb.GGML_Q4_K, qk(KVD, HID)), (bb.GGML_Q6_K, qk(KVD, HID, True)),
                       (bb.GGML_Q4_K, qk(HID, HID)), qg, kg, device=dev.index)
    g = torch.Generator(device=dev)
    g.manual_seed(8)
    x = 0.5 * torch.randn((T, HID), generator=g, device=dev)
    xs = 0.5 * torch.randn((steps, HID), generator=g, device=dev)
    out = torch.empty((T, HID), device=dev)
    o1 = torch.empty(HID, device=dev)
    # both caches draw from one pool: the warm-up call sizes the pool's scratch, so the timed
    # call allocates nothing
    pool = bb.Pool(n_layers=1, n_pages=2 * ((T + 3 * steps) // 64 + 4), device=dev.index)
    caches = [bb.Cache(max_context=T + 3 * steps + 64, pool=pool) for _ in range(2)]
    e = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    for rep, c in enumerate(caches):  # the first is the warm-up
        torch.cuda.synchronize()
        e[0].record(stream)
        bb.attn_layer_batch(c, 0, W, x, 0, tensor_cores=True, theta=THETA, out=out, stream=stream)
        e[1].record(stream)
        for s_ in range(steps):
            bb.attn_layer_step(c, 0, W, xs[s_], T + s_, theta=THETA, out=o1, stream=stream)
        e[2].record(stream)
        torch.cuda.synchronize()
    batch_ms, step_ms = e[0].elapsed_time(e[1]), e[1].elapsed_time(e[2]) / steps
    # the same single-token steps as one CUDA graph: a whole-operator step plan, `steps` tokens
    # captured once (each node reads its own token's input), replayed twice (warm-up, timed)
    c = caches[1]
    c.pos = T + steps
    plan = bb.StepPlan(c, 0, weights=W)
    graph, cap = torch.cuda.CUDAGraph(), torch.cuda.Stream()
    torch.cuda.synchronize()
    with torch.cuda.graph(graph, stream=cap):
        for s_ in range(steps):
            plan.launch_layer(xs[s_], o1, theta=THETA)
    graph.replay()
    torch.cuda.synchronize()
    e[0].record(stream)
    graph.replay()
    e[1].record(stream)
    torch.cuda.synchronize()
    graph_step_ms = e[0].elapsed_time(e[1]) / steps
    plan.finish()
    for c in caches:
        c.close()
    pool.close()
    W.close()
    proj_macs = (2 * HID * HID + 2 * KVD * HID) * T
    return {"workload": f"attention operator of one layer: {T}-token chunk (Q4_K/Q6_K projections + tensor-core "
                        f"prefill + output projection), then {steps} single-token steps",
            "batch_ms": round(batch_ms, 3), "batch_tok_per_s": round(T / (batch_ms * 1e-3), 1),
            "projection_tmacs_per_s_upper_bound": round(proj_macs / (batch_ms * 1e-3) / 1e12, 2),
            "step_ms": round(step_ms, 4), "step_tok_per_s": round(1 / (step_ms * 1e-3), 1),
            "graph_step_ms": round(graph_step_ms, 4),
            "graph_how": "whole-operator step plan, all steps captured in one CUDA graph"}


def bench_logits_head(bb, torch, dev, stream, hbm_peak, peak_kind, vocab=128000, steps=50):
    """The logits head (src/model.rs:379-388) and greedy token (src/sampler.rs:139-149) per
    decode token, on the device: RMSNorm, the tied token_embd matvec (synthetic Q6_K,
    [128000][2048] = 215 MB, read once per token; larger than L2) and argmax."""
    import numpy as np
    rng = np.random.default_rng(11)
    nb = HID // 256
    w = rng.integers(0, 256, size=(vocab, nb, 210), dtype=np.uint8)
    w[:, :, 208:210] = (rng.standard_normal((vocab, nb)) * 0.002).astype(np.float16).view(np.uint8).reshape(vocab, nb, 2)
    head = bb.Head(bb.GGML_Q6_K, w.reshape(-1), HID, vocab, np.ones(HID, np.float32), device=dev.index)
    del w
    g = torch.Generator(device=dev)
    g.manual_seed(12)
    hs = torch.randn((steps, HID), generator=g, device=dev)
    tok = torch.zeros(1, dtype=torch.int32, device=dev)
    lib = bb.load_library()
    sp = stream.cuda_stream
    for i in range(3):
        lib.bebelm_head_logits(head._h, hs[i].data_ptr(), 1e-5, None, tok.data_ptr(), bb.MEM_DEVICE, sp)
    e = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    torch.cuda.synchronize()
    e[0].record(stream)
    for i in range(steps):
        lib.bebelm_head_logits(head._h, hs[i].data_ptr(), 1e-5, None, tok.data_ptr(), bb.MEM_DEVICE, sp)
    e[1].record(stream)
    torch.cuda.synchronize()
    head.close()
    ms = e[0].elapsed_time(e[1]) / steps
    wbytes = vocab * nb * 210
    gbs = wbytes / (ms * 1e-3) / 1e9
    return {"workload": f"logits head per decode token: RMSNorm + Q6_K token_embd [{vocab}][{HID}] matvec + argmax, "
                        "device in/out, one launch (norm, matvec and argmax fused)",
            "ms_per_token": round(ms, 4), "weight_gbs": round(gbs, 1),
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm_peak, "unit": "GB/s",
                         "frac": round(gbs / hbm_peak, 4), "peak_kind": peak_kind}}


def bench_config3_narrow(bb, torch, dev, stream, world, steps, kv_dtype):
    """Config 3 with a bf16 or fp8 (e4m3) KV cache: same step, a half or a quarter of the bytes
    per position."""
    cache = bb.Cache(n_layers=1, max_context=CTX, device=dev.index, kv_dtype=kv_dtype)
    g = torch.Generator(device=dev)
    g.manual_seed(31)
    for c0 in range(0, CTX, 4096):
        cache.append(0, torch.randn((4096, KVD), generator=g, device=dev), torch.randn((4096, KVD), generator=g, device=dev))
    n = steps + 5
    Q = torch.randn((n, HID), generator=g, device=dev)
    K = torch.randn((n, KVD), generator=g, device=dev)
    V = torch.randn((n, KVD), generator=g, device=dev)
    qg = 1 + 0.02 * torch.randn(D, generator=g, device=dev)
    kg = 1 + 0.02 * torch.randn(D, generator=g, device=dev)
    out = torch.empty((n, HID), device=dev)
    for i in range(5):
        cache.attn_step(0, Q[i], K[i], V[i], qg, kg, pos=CTX + i, theta=THETA, out=out[i], stream=stream)
        cache.evict_front(1)
    barrier(world)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for i in range(5, n):
        cache.attn_step(0, Q[i], K[i], V[i], qg, kg, pos=CTX + i, theta=THETA, out=out[i], stream=stream)
        cache.evict_front(1)
    b.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(a.elapsed_time(b), world, dev)
    cache.close()
    es, name = (2, "bf16") if kv_dtype == bb.BF16 else (1, "fp8 e4m3")
    per_step = 2 * (CTX + 1) * KVD * es
    return {"workload": f"config3 with a {name} KV cache (K/V rounded on append, attention in fp32)",
            "value": round(per_step * steps * world / (ms * 1e-3) / 1e9, 1), "unit": f"GB/s ({name} bytes)",
            "tok_per_s": round(steps * world / (ms * 1e-3), 1), "ms_per_step": round(ms / steps, 5)}


def bench_config4(bb, torch, dev, stream, world, rank, steps=128):
    """Config 4: 64 independent sequences, KV lengths U[1024, 16384] by seed, one decode token
    each per step, sequences LPT-sharded over the ranks (no collective)."""
    import numpy as np
    from bebelm_b200.sharded import assign_sequences
    lengths = np.random.default_rng(4).integers(1024, 16385, size=64)
    mine = assign_sequences(lengths, world)[rank]
    pages = sum(int(lengths[i]) // 64 + (steps + 72) // 64 + 3 for i in mine)
    pool = bb.Pool(n_layers=1, n_pages=pages, device=dev.index)
    caches = [bb.Cache(max_context=int(lengths[i]) + steps + 72, pool=pool) for i in mine]
    g = torch.Generator(device=dev)
    g.manual_seed(40 + rank)
    for c, i in zip(caches, mine):
        for c0 in range(0, int(lengths[i]), 8192):
            n = min(8192, int(lengths[i]) - c0)
            c.append(0, torch.randn((n, KVD), generator=g, device=dev), torch.randn((n, KVD), generator=g, device=dev))
    n = len(mine)
    WARM4 = 8  # untimed steps first (the pool's pages are touched for the first time there)
    Q = torch.randn((steps + WARM4, n, HID), generator=g, device=dev)
    K = torch.randn((steps + WARM4, n, KVD), generator=g, device=dev)
    V = torch.randn((steps + WARM4, n, KVD), generator=g, device=dev)
    qg = 1 + 0.02 * torch.randn(D, generator=g, device=dev)
    kg = 1 + 0.02 * torch.randn(D, generator=g, device=dev)
    out = torch.empty((n, HID), device=dev)
    pos = [int(lengths[i]) for i in mine]
    for i in range(WARM4):
        bb.attn_decode_batched(caches, 0, Q[i], K[i], V[i], qg, kg, pos, theta=THETA, out=out, stream=stream)
        pos = [p + 1 for p in pos]
    barrier(world)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for i in range(WARM4, steps + WARM4):
        bb.attn_decode_batched(caches, 0, Q[i], K[i], V[i], qg, kg, pos, theta=THETA, out=out, stream=stream)
        pos = [p + 1 for p in pos]
    b.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    ms_local = a.elapsed_time(b)
    if os.environ.get("BEBELM_BENCH_VERBOSE"):
        print(f"config4 rank {rank}: {len(mine)} seqs, {sum(int(lengths[i]) for i in mine)} positions, "
              f"{ms_local / steps:.4f} ms/step", file=sys.stderr, flush=True)
    ms = max_over_ranks(ms_local, world, dev)
    total = sum(bytes_per_step(int(l) + WARM4 + s + 1) for l in lengths for s in range(steps))
    for c in caches:
        c.close()
    pool.close()
    return {"workload": "config4: 64 sequences, KV lengths U[1024,16384] (seed 4), 128 decode steps, 64-token pages",
            "value": round(total / (ms * 1e-3) / 1e9, 1), "unit": "GB/s",
            "tok_per_s": round(64 * steps / (ms * 1e-3), 1), "ms_per_step": round(ms / steps, 4),
            "parallelism": f"per-sequence x{world} (LPT by KV length), no collective"}


def bench_config5(bb, torch, dev, stream, world, rank, bf16_peak, T=8192, steps=512):
    """Config 5: the 6 attention layers of the stack, KV heads sharded over the ranks: causal
    prefill of T bf16 tokens whose all-gather of head outputs is fused into the prefill kernel's
    epilogue, then `steps` decode steps whose all-gather is fused into the decode kernel (both:
    tagged 8-byte words stored over NVLink into every rank's landing zone). Decode is timed
    host-driven and as one CUDA graph of step plans (all steps x 6 layers). With more than one
    rank, rank 0 also runs the same workload unsharded on its own GPU (the others wait), so the
    line carries the 1 -> N speed-up and efficiency of this run; the host-driven decode is also
    timed with an NCCL all-gather instead of the fused one, for comparison."""
    from bebelm_b200.sharded import KVHeadSharded
    L = 6
    g = torch.Generator(device=dev)
    g.manual_seed(50)  # identical activations on every rank (replicated projections)
    q = torch.randn((T, HID), generator=g, device=dev).to(torch.bfloat16)
    k = torch.randn((T, KVD), generator=g, device=dev).to(torch.bfloat16)
    v = torch.randn((T, KVD), generator=g, device=dev).to(torch.bfloat16)
    qg = 1 + 0.02 * torch.randn(D, generator=g, device=dev)
    kg = 1 + 0.02 * torch.randn(D, generator=g, device=dev)
    Qd = torch.randn((steps, HID), generator=g, device=dev)
    Kd = torch.randn((steps, KVD), generator=g, device=dev)
    Vd = torch.randn((steps, KVD), generator=g, device=dev)

    def ev():
        return torch.cuda.Event(enable_timing=True)

    def run(sh, sync):
        """prefill ms, host-driven decode ms, graph decode ms (per whole run, this rank)."""
        for layer in range(L):  # untimed warm-up of every call and collective the timed region makes
            sh.attn_prefill(layer, q, k, v, qg, kg, 0, theta=THETA)
            for s_ in range(3):
                sh.attn_step(layer, Qd[s_], Kd[s_], Vd[s_], qg, kg, pos=T + s_, theta=THETA)
        sh.clear()
        sync()
        e = [ev() for _ in range(3)]
        e[0].record(stream)
        for layer in range(L):
            sh.attn_prefill(layer, q, k, v, qg, kg, 0, theta=THETA)
        e[1].record(stream)
        for s_ in range(steps):
            for layer in range(L):
                sh.attn_step(layer, Qd[s_], Kd[s_], Vd[s_], qg, kg, pos=T + s_, theta=THETA)
        e[2].record(stream)
        torch.cuda.synchronize()
        sync()
        pre, dec = e[0].elapsed_time(e[1]), e[1].elapsed_time(e[2])
        if getattr(sh, "peers", 1) is None and sh.world > 1:
            return pre, dec, None
        # decode as one CUDA graph: a step plan per layer, all `steps` x 6 layers captured once
        # (each node reads its own step's inputs) and replayed twice (warm-up, timed)
        sh.clear()
        for layer in range(L):
            sh.attn_prefill(layer, q, k, v, qg, kg, 0, theta=THETA)
        sh.cache.pos = T
        plans = sh.step_plans()
        o = torch.empty((steps, L, HID), device=dev)
        graph, cap = torch.cuda.CUDAGraph(), torch.cuda.Stream()
        torch.cuda.synchronize()
        with torch.cuda.graph(graph, stream=cap, capture_error_mode="thread_local"):  # NCCL watchdog threads run meanwhile
            for s_ in range(steps):
                for layer in range(L):
                    sh.plan_step(plans[layer], Qd[s_], Kd[s_], Vd[s_], qg, kg, o[s_, layer], theta=THETA)
        sync()
        graph.replay()
        torch.cuda.synchronize()
        sync()
        e = [ev() for _ in range(2)]
        e[0].record(stream)
        graph.replay()
        e[1].record(stream)
        torch.cuda.synchronize()
        sync()
        for p_ in plans:
            p_.finish()
        sh.cache.check()
        return pre, dec, e[0].elapsed_time(e[1])

    flops = L * 4096.0 * T * (T + 1)

    def line(pre, dec, gms, n):
        tf = flops / (pre * 1e-3) / 1e12
        out = {"prefill_ms": round(pre, 3), "prefill_tflops": round(tf, 1),
               "prefill_frac_of_bf16_peak_per_gpu": round(tf / n / bf16_peak, 4),
               "decode_ms_per_step": round(dec / steps, 4), "decode_tok_per_s": round(steps / (dec * 1e-3), 1)}
        if gms is not None:
            out["decode_graph"] = {"ms_per_step": round(gms / steps, 4), "tok_per_s": round(steps / (gms * 1e-3), 1),
                                   "how": "step plans, one CUDA graph of all steps x 6 layers"}
        return out

    sync = (lambda: barrier(world))
    sh = KVHeadSharded(n_layers=L, max_context=T + 2 * steps + 64)
    pre, dec, gms = run(sh, sync)
    sh.close()
    sh.cache.close()
    pre = max_over_ranks(pre, world, dev)
    dec = max_over_ranks(dec, world, dev)
    gms = max_over_ranks(gms, world, dev)
    out = {"workload": f"config5: 6 GQA layers, causal prefill of {T} bf16 tokens then {steps} decode steps",
           **line(pre, dec, gms, world),
           "parallelism": (f"kv heads / {world} per GPU; all-gather of head outputs fused into the prefill "
                           "and decode kernels (tagged words stored over NVLink)") if world > 1
           else "one GPU, all heads"}
    if world > 1:
        shn = KVHeadSharded(n_layers=L, max_context=T + 2 * steps + 64, fused_gather=False)
        _, dec_nccl, _ = run(shn, sync)
        shn.close()
        shn.cache.close()
        out["decode_ms_per_step_nccl_gather"] = round(max_over_ranks(dec_nccl, world, dev) / steps, 4)
        # the same workload unsharded on rank 0's GPU (one process, no collective) in this run
        base = None
        if rank == 0:
            one = KVHeadSharded(n_layers=L, max_context=T + 2 * steps + 64, local=True)
            b_pre, b_dec, b_g = run(one, lambda: None)
            one.cache.close()
            base = line(b_pre, b_dec, b_g, 1)
            out["one_gpu_same_run"] = base
            out["speedup_vs_1gpu"] = {
                "prefill": round(b_pre / pre, 3), "decode_graph": round(b_g / gms, 3),
                "decode_host_driven": round(b_dec / dec, 3)}
            out["efficiency_vs_1gpu"] = {k_: round(v_ / world, 3) for k_, v_ in out["speedup_vs_1gpu"].items()}
        barrier(world)
    return out


def profile_workload(name: str):
    """Small cases for ncu captures of one kernel each (inputs above L2 where it matters, a few
    GB at most): `norm_rope` (config-2 prefill: kernel 1 then the tensor-core prefill), `batched`
    (batched decode over 16 sequences of U[1024,16384] positions, ~560 MB of fp32 K/V),
    `qmv` (one-token attention operator steps: the qmv_lane_kernel projections), `aux` (the
    small kernels around them: host-buffer decode steps on a 32768-position window, whose
    inputs a stage_copy_kernel brings in; a 2048-token prefill chunk after 6144 cached positions,
    whose prefix kv_gather_bf16_kernel gathers; fused all-gather steps through a one-rank peer
    group, whose words gather_ll_kernel copies out)."""
    import numpy as np
    import torch
    import bebelm_b200 as bb
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    qg = torch.ones(D, device=dev)
    if name == "norm_rope":
        T = 2048
        q = torch.randn((T, HID), generator=g, device=dev).to(torch.bfloat16)
        k = torch.randn((T, KVD), generator=g, device=dev).to(torch.bfloat16)
        v = torch.randn((T, KVD), generator=g, device=dev).to(torch.bfloat16)
        for _ in range(3):
            c = bb.Cache(n_layers=1, max_context=T)
            c.attn_prefill(0, q, k, v, qg, qg, 0, theta=THETA)
            torch.cuda.synchronize()
            c.close()
    elif name == "batched":
        lengths = np.random.default_rng(4).integers(1024, 16385, size=16)
        pool = bb.Pool(n_layers=1, n_pages=sum(int(l) // 64 + 4 for l in lengths))
        cs = [bb.Cache(max_context=int(l) + 64, pool=pool) for l in lengths]
        for c, l in zip(cs, lengths):
            c.append(0, torch.randn((int(l), KVD), generator=g, device=dev),
                     torch.randn((int(l), KVD), generator=g, device=dev))
        Q = torch.randn((16, HID), generator=g, device=dev)
        K = torch.randn((16, KVD), generator=g, device=dev)
        for s_ in range(3):
            bb.attn_decode_batched(cs, 0, Q, K, K, qg, qg, [int(l) + s_ for l in lengths], theta=THETA)
        torch.cuda.synchronize()
        for c in cs:
            c.close()
        pool.close()
    elif name == "qmv":
        rng = np.random.default_rng(3)

        def kq(rows, n_in, six=False):
            nb = 210 if six else 144
            w = rng.integers(0, 256, size=(rows, n_in // 256, nb), dtype=np.uint8)
            d = (rng.standard_normal((rows, n_in // 256)) * (0.002 if six else 0.01)).astype(np.float16)
            w[:, :, (208 if six else 0):(210 if six else 2)] = d.view(np.uint8).reshape(rows, -1, 2)
            return w.reshape(-1)

        W = bb.AttnWeights((bb.GGML_Q4_K, kq(HID, HID)), (bb.GGML_Q4_K, kq(KVD, HID)),
                           (bb.GGML_Q6_K, kq(KVD, HID, True)), (bb.GGML_Q4_K, kq(HID, HID)),
                           np.ones(D, np.float32), np.ones(D, np.float32))
        c = bb.Cache(n_layers=1, max_context=4096)
        c.append(0, torch.randn((2000, KVD), generator=g, device=dev), torch.randn((2000, KVD), generator=g, device=dev))
        x = torch.randn((8, HID), generator=g, device=dev)
        o = torch.empty(HID, device=dev)
        for i in range(8):
            bb.attn_layer_step(c, 0, W, x[i], 2000 + i, theta=THETA, out=o)
        torch.cuda.synchronize()
    elif name == "aux":
        c = bb.Cache(n_layers=1, max_context=CTX)
        for c0 in range(0, CTX, 4096):
            c.append(0, torch.randn((4096, KVD), generator=g, device=dev), torch.randn((4096, KVD), generator=g, device=dev))
        c.evict_front(1)
        rng = np.random.default_rng(6)
        qh, kh, vh = (rng.standard_normal(n, dtype=np.float32) for n in (HID, KVD, KVD))
        gh = np.ones(D, np.float32)
        for i in range(4):  # host buffers: the inputs come in through the staging copy kernel
            c.attn_step(0, qh, kh, vh, gh, gh, pos=CTX + i, theta=THETA)
            c.evict_front(1)
        c.close()
        T0, T1 = 6144, 2048
        q = torch.randn((T0 + T1, HID), generator=g, device=dev).to(torch.bfloat16)
        k = torch.randn((T0 + T1, KVD), generator=g, device=dev).to(torch.bfloat16)
        c = bb.Cache(n_layers=1, max_context=T0 + T1)
        c.attn_prefill(0, q[:T0], k[:T0], k[:T0], qg, qg, 0, theta=THETA)
        c.attn_prefill(0, q[T0:], k[T0:], k[T0:], qg, qg, T0, theta=THETA)  # gathers the 6144 cached positions
        torch.cuda.synchronize()
        c.close()
        c = bb.Cache(n_layers=1, max_context=4096)
        c.append(0, torch.randn((4000, KVD), generator=g, device=dev), torch.randn((4000, KVD), generator=g, device=dev))
        grp = bb.PeerGroup(1, 0, HID, device=0)
        grp.connect([grp.handle])
        x = torch.randn((3, HID), generator=g, device=dev)
        kx = torch.randn((3, KVD), generator=g, device=dev)
        for i in range(3):
            c.attn_step_allgather(grp, 0, x[i], kx[i], kx[i], qg, qg, pos=4000 + i, theta=THETA)
        torch.cuda.synchronize()
        c.check()
        grp.close()
        c.close()
    else:
        raise SystemExit(f"unknown profile workload {name}")
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--no-cfg4", action="store_true")
    ap.add_argument("--no-cfg5", action="store_true")
    ap.add_argument("--profile-workload", default=None, choices=["norm_rope", "batched", "qmv", "aux"],
                    help="run one small case for an ncu capture and exit")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.profile_workload:
        return profile_workload(args.profile_workload)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
