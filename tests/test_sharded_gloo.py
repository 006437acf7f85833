"""Host logic of the multi-GPU layouts, on gloo ranks (CPU only).

Each rank runs its KV-head shard through an oracle-backed cache; the all-gathered output
must equal the unsharded oracle exactly (heads are independent). The CUDA path runs the
same KVHeadSharded code with the device cache and NCCL (bench.py --gpus N).
"""
import multiprocessing as mp
import os
import socket

import numpy as np
import pytest
import torch

import oracle
from bebelm_b200.sharded import KVHeadSharded, assign_sequences

H, KVH, D = 32, 8, 64


class OracleShardCache:
    """The cache interface KVHeadSharded drives, on the CPU oracle (one shard of kv heads)."""

    def __init__(self, n_layers, n_kv, max_context):
        self.n_kv = n_kv
        self.c = oracle.Cache(n_layers, n_kv * D)

    def attn_step(self, layer, q, k, v, q_gain, k_gain, pos, theta, eps):
        n_heads = q.numel() // D
        out = self.c.attn_step(layer, q.numpy(), k.numpy(), v.numpy(), q_gain.numpy(), k_gain.numpy(), theta, eps,
                               n_heads, self.n_kv, D, pos=pos)
        return torch.from_numpy(out)

    def attn_prefill(self, layer, q, k, v, q_gain, k_gain, pos0, theta, eps, n_heads):
        ck = self.c.k[layer] if self.c.k[layer].shape[0] else None
        cv = self.c.v[layer] if self.c.v[layer].shape[0] else None
        out, nk, nv, _, _ = oracle.attn_batch(q.numpy(), k.numpy(), v.numpy(), pos0, q_gain.numpy(), k_gain.numpy(),
                                              theta, eps, n_heads, self.n_kv, D, ck, cv)
        self.c.k[layer], self.c.v[layer] = nk, nv
        return torch.from_numpy(out)

    def evict_front(self, n):
        self.c.evict_front(n)

    def kv_len(self):
        return self.c.kv_len()

    def clear(self):
        self.c = oracle.Cache(len(self.c.k), self.n_kv * D)


def _inputs(seed, t):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn((t, H * D), generator=g), torch.randn((t, KVH * D), generator=g),
            torch.randn((t, KVH * D), generator=g), 1 + 0.02 * torch.randn(D, generator=g),
            1 + 0.02 * torch.randn(D, generator=g))


def _worker(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.distributed.init_process_group("gloo", rank=rank, world_size=world)
        sh = KVHeadSharded(n_layers=2, max_context=1024, cache_factory=OracleShardCache)
        qq, kk, vv, qg, kg = _inputs(5, 40)
        pre = sh.attn_prefill(1, qq[:32], kk[:32], vv[:32], qg, kg, 0, 1e6, 1e-5)
        steps = [sh.attn_step(1, qq[32 + i], kk[32 + i], vv[32 + i], qg, kg, 32 + i, 1e6, 1e-5) for i in range(8)]
        sh.evict_front(5)
        after = sh.attn_step(1, qq[0], kk[1], vv[2], qg, kg, 40, 1e6, 1e-5)
        q.put((rank, pre.numpy(), np.stack([s.numpy() for s in steps]), after.numpy(), sh.kv_len()))
        torch.distributed.destroy_process_group()
    except Exception as e:  # surface the failure to the parent
        q.put((rank, repr(e), None, None, None))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 4])
def test_kv_head_sharding_matches_unsharded(world):
    ctx = mp.get_context("fork")
    q = ctx.Queue()
    port = _free_port()
    # daemon ranks, ended on the way out: a rank that hangs (e.g. forked from a process that
    # had initialised CUDA) must not keep the interpreter from exiting
    procs = [ctx.Process(target=_worker, args=(r, world, port, q), daemon=True) for r in range(world)]
    for p in procs:
        p.start()
    try:
        res = [q.get(timeout=180) for _ in range(world)]
        for p in procs:
            p.join(timeout=60)
    finally:
        for p in procs:
            if p.is_alive():
                p.terminate()
    for r in res:
        assert not isinstance(r[1], str), r[1]
    # unsharded reference
    full = OracleShardCache(2, KVH, 1024)
    qq, kk, vv, qg, kg = _inputs(5, 40)
    pre = full.attn_prefill(1, qq[:32], kk[:32], vv[:32], qg, kg, 0, 1e6, 1e-5, H).numpy()
    steps = np.stack([full.attn_step(1, qq[32 + i], kk[32 + i], vv[32 + i], qg, kg, 32 + i, 1e6, 1e-5).numpy()
                      for i in range(8)])
    full.evict_front(5)
    after = full.attn_step(1, qq[0], kk[1], vv[2], qg, kg, 40, 1e6, 1e-5).numpy()
    for rank, p_, s_, a_, n in res:
        assert np.array_equal(p_, pre) and np.array_equal(s_, steps) and np.array_equal(a_, after), rank
        assert n == full.kv_len()


def test_assign_sequences_lpt():
    lengths = oracle.uniform_int(3, 64, 1024, 16384)
    for world in (1, 2, 4, 8):
        parts = assign_sequences(lengths, world)
        flat = sorted(i for p in parts for i in p)
        assert flat == list(range(64))
        loads = [int(sum(lengths[i] for i in p)) for p in parts]
        assert max(loads) - min(loads) <= int(lengths.max())  # LPT bound
