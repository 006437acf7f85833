"""Multi-GPU layouts of the attention path (one process per GPU, torch.distributed).

* :class:`KVHeadSharded` — KV-head sharding. Rank r of N owns kv heads
  [8r/N, 8(r+1)/N) and their query heads [32r/N, 32(r+1)/N) for every attention
  layer; its cache holds only those heads, so each rank reads 1/N of the KV bytes.
  The head outputs are gathered inside the kernels (``fused_gather``): the CTAs
  that finish a head (decode) or a tile of query rows (tensor-core prefill) store
  it into every rank's landing zone over NVLink as words tagged with the step's
  number, which the receiving rank polls (:class:`bebelm_b200.PeerGroup`); other
  prefills all-gather over NCCL. Rank order is head order, so the gathered buffer
  is the full [n_heads*64] (or [t, n_heads*64]) output of ``attn_step`` /
  ``attn_batch`` (src/model.rs:440-451, 232-254).
* :func:`assign_sequences` — per-sequence sharding for independent Agent
  sequences: longest-processing-time assignment of sequences to ranks by KV
  length. No collective is needed; each rank runs batched decode on its share.

The per-rank cache defaults to :class:`bebelm_b200.Cache` on the current CUDA
device; ``cache_factory`` lets a test substitute another implementation of the
same methods (e.g. a CPU reference) to check the sharding and gather logic on
gloo ranks.
"""
from __future__ import annotations

import heapq

import torch
import torch.distributed as dist

from . import HEAD_DIM, N_HEADS, N_KV_HEADS, RMS_EPS, ROPE_THETA, Cache, PeerGroup


def assign_sequences(lengths, world: int):
    """Longest-processing-time assignment: sequence indices per rank, balancing the summed
    KV lengths (the bytes each rank's decode reads)."""
    heap = [(0, r) for r in range(world)]
    out = [[] for _ in range(world)]
    for i in sorted(range(len(lengths)), key=lambda i: -int(lengths[i])):
        load, r = heapq.heappop(heap)
        out[r].append(i)
        heapq.heappush(heap, (load + int(lengths[i]), r))
    return [sorted(x) for x in out]


class KVHeadSharded:
    """One rank's share of a KV-head-sharded attention stack."""

    def __init__(self, n_layers: int, max_context: int, n_heads: int = N_HEADS, n_kv_heads: int = N_KV_HEADS,
                 group=None, cache_factory=None, fused_gather: bool | None = None, local: bool = False,
                 max_prefill_tokens: int = 8192):
        """fused_gather: gather decode outputs inside the decode kernel over peer memory, and
        tensor-core prefill outputs (chunks up to max_prefill_tokens) inside the prefill kernel
        (default: on for the CUDA cache with more than one rank); off uses NCCL. local: this
        process alone holds every head (world 1), whatever the process group."""
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() and not local else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() and not local else 0
        if n_kv_heads % self.world or n_heads % n_kv_heads:
            raise ValueError(f"{n_kv_heads} kv heads cannot be split over {self.world} ranks")
        self.n_heads, self.n_kv = n_heads, n_kv_heads
        self.kv_per = n_kv_heads // self.world
        self.h_per = n_heads // self.world
        self.h0, self.kv0 = self.rank * self.h_per, self.rank * self.kv_per
        if cache_factory is None:
            dev = torch.cuda.current_device()
            self.cache = Cache(n_layers=n_layers, n_kv_heads=self.kv_per, max_context=max_context, device=dev)
        else:
            self.cache = cache_factory(n_layers, self.kv_per, max_context)
        if fused_gather is None:
            fused_gather = cache_factory is None and self.world > 1
        self.peers = self.prefill_peers = None
        self.max_prefill_tokens = max_prefill_tokens
        if fused_gather:
            dev = torch.cuda.current_device()
            self.peers = PeerGroup(self.world, self.rank, self.h_per * HEAD_DIM, device=dev)
            self.prefill_peers = PeerGroup(self.world, self.rank, max_prefill_tokens * self.h_per * HEAD_DIM, device=dev)
            for g in (self.peers, self.prefill_peers):
                handles = [None] * self.world
                dist.all_gather_object(handles, g.handle, group=self.group)
                g.connect(handles)
            dist.barrier(group=self.group)

    # -- slicing ---------------------------------------------------------------
    def _heads(self, x, per, first, t=None):
        if self.world == 1:
            return x
        if t is None:  # consecutive heads of one token: a contiguous view
            return x.reshape(-1)[first * HEAD_DIM:(first + per) * HEAD_DIM]
        return x.reshape(t, -1, HEAD_DIM)[:, first:first + per].reshape(t, -1).contiguous()

    def _gather(self, local):
        if self.world == 1:
            return local
        local = local.contiguous()
        flat = local.new_empty(self.world * local.numel())  # concatenated in rank order
        dist.all_gather_into_tensor(flat, local.reshape(-1), group=self.group)
        return flat.view((self.world,) + tuple(local.shape))

    # -- the reference operator ------------------------------------------------
    def attn_step(self, layer: int, q, k, v, q_gain, k_gain, pos: int, theta: float = ROPE_THETA,
                  eps: float = RMS_EPS):
        """q [n_heads*64], k/v [n_kv*64] (replicated on every rank) -> full out [n_heads*64]."""
        if self.peers is not None:
            return self.cache.attn_step_allgather(self.peers, layer, self._heads(q, self.h_per, self.h0),
                                                  self._heads(k, self.kv_per, self.kv0),
                                                  self._heads(v, self.kv_per, self.kv0), q_gain, k_gain, pos=pos,
                                                  theta=theta, eps=eps)
        out = self.cache.attn_step(layer, self._heads(q, self.h_per, self.h0), self._heads(k, self.kv_per, self.kv0),
                                   self._heads(v, self.kv_per, self.kv0), q_gain, k_gain, pos=pos, theta=theta, eps=eps)
        return self._gather(out).reshape(-1)

    def attn_prefill(self, layer: int, q, k, v, q_gain, k_gain, pos0: int, theta: float = ROPE_THETA,
                     eps: float = RMS_EPS):
        """q [t, n_heads*64], k/v [t, n_kv*64] -> full out [t, n_heads*64]."""
        t = q.shape[0]
        if self.prefill_peers is not None and t <= self.max_prefill_tokens and q.dtype == torch.bfloat16:
            # the tensor-core prefill stores every rank's rows into every landing zone itself
            return self.cache.attn_prefill_allgather(self.prefill_peers, layer, q.contiguous(), k.contiguous(),
                                                     v.contiguous(), q_gain, k_gain, pos0, theta=theta, eps=eps,
                                                     n_heads=self.h_per)
        out = self.cache.attn_prefill(layer, self._heads(q, self.h_per, self.h0, t),
                                      self._heads(k, self.kv_per, self.kv0, t), self._heads(v, self.kv_per, self.kv0, t),
                                      q_gain, k_gain, pos0, theta=theta, eps=eps, n_heads=self.h_per)
        full = self._gather(out)  # [world, t, h_per*64]
        if self.world == 1:
            return full
        return full.permute(1, 0, 2).reshape(t, -1)

    def step_plans(self, window: int = 0) -> list:
        """One device-driven step plan per layer of this rank's cache (see
        :class:`bebelm_b200.StepPlan`), for decode steps captured in a CUDA graph."""
        return [self.cache.step_plan(layer, n_heads=self.h_per, window=window)
                for layer in range(self.cache.n_layers)]

    def plan_step(self, plan, q, k, v, q_gain, k_gain, out, theta: float = ROPE_THETA, eps: float = RMS_EPS):
        """One step of ``plan`` (a :meth:`step_plans` entry): q [n_heads*64], k/v [n_kv*64]
        replicated -> out [n_heads*64], gathered inside the step (fused) with no host work, so
        the call can be captured in a CUDA graph on every rank."""
        q, k, v = (self._heads(x, per, first).contiguous() for x, per, first in
                   ((q, self.h_per, self.h0), (k, self.kv_per, self.kv0), (v, self.kv_per, self.kv0)))
        if self.peers is None:
            if self.world > 1:
                raise RuntimeError("plan steps on several ranks need the fused gather")
            return plan.launch(q, k, v, q_gain, k_gain, out, theta=theta, eps=eps)
        return plan.launch_allgather(self.peers, q, k, v, q_gain, k_gain, out, theta=theta, eps=eps)

    def evict_front(self, n: int):
        self.cache.evict_front(n)

    def kv_len(self) -> int:
        return self.cache.kv_len()

    def clear(self):
        self.cache.clear()

    def close(self):
        """Collective: every rank's steps are done before any landing zone is freed."""
        if self.peers is not None:
            torch.cuda.synchronize()
            dist.barrier(group=self.group)
            self.peers.close()
            self.prefill_peers.close()
            self.peers = self.prefill_peers = None
