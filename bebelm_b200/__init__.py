"""bebelm_b200 — B200 (sm_100a) attention hot path for BebeLM, behind a C-ABI.

Python mirror of the reference's attention interface, calling the in-tree CUDA
library ``libbebelm_attn.so`` through ctypes:

* :func:`attention_decode` — ``attention_decode`` (src/kernels/attention.rs:17-26)
* :func:`norm_rope_heads` — ``norm_rope_heads`` (src/model.rs:600-608)
* :class:`Cache` — the attention part of ``Cache`` (src/cache.rs:9-49) as a
  device-resident paged window, with ``attn_step`` (src/model.rs:440-451),
  ``attn_prefill`` (src/model.rs:232-254) and batched decode across caches of
  one :class:`Pool`.

Host buffers are numpy float32 arrays; device buffers are CUDA torch tensors
(their data pointers are passed as-is). There is no CPU fallback: if the
library is missing or no sm_100 device is visible, calls raise.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libbebelm_attn.so")

OK, ERR_INVALID, ERR_CUDA, ERR_OOM, ERR_CAPACITY, ERR_UNSUPPORTED, ERR_TIMEOUT, ERR_NO_DEVICE = 0, -1, -2, -3, -4, -5, -7, -8
ERR_FORMAT, ERR_NOT_FOUND, ERR_IO = -9, -10, -11
MEM_HOST, MEM_DEVICE = 0, 1
F32, BF16 = 0, 1
F32_TENSOR = 2  # prefill in_dtype: fp32 inputs, tensor-core attention
FP8 = 3  # cache dtype: K/V as fp8 e4m3

# reference constants (src/config.rs:14-32)
N_HEADS, N_KV_HEADS, HEAD_DIM, KV_DIM, HIDDEN = 32, 8, 64, 512, 2048
ROPE_THETA, RMS_EPS = 5_000_000.0, 1e-5
ATTENTION_LAYERS = (2, 6, 10, 14, 18, 21)

EXPORTS = [
    "bebelm_abi_version", "bebelm_last_error", "bebelm_device_count", "bebelm_attn_decode_host",
    "bebelm_norm_rope_heads", "bebelm_kv_pool_create", "bebelm_kv_pool_destroy", "bebelm_kv_pool_free_pages",
    "bebelm_kv_create", "bebelm_kv_create_in_pool", "bebelm_kv_destroy", "bebelm_kv_clone", "bebelm_kv_clear",
    "bebelm_kv_len", "bebelm_kv_layer_len", "bebelm_kv_pos", "bebelm_kv_set_pos", "bebelm_kv_evict_front",
    "bebelm_kv_append", "bebelm_kv_read", "bebelm_attn_step", "bebelm_attn_decode_cached", "bebelm_attn_decode_cached_noalloc", "bebelm_attn_prefill", "bebelm_attn_decode_batched",
    "bebelm_kv_check", "bebelm_debug_expire_next_wait", "bebelm_peer_group_create", "bebelm_peer_group_connect", "bebelm_peer_group_destroy",
    "bebelm_attn_step_allgather", "bebelm_step_plan_create", "bebelm_step_plan_launch", "bebelm_step_plan_steps",
    "bebelm_step_plan_finish", "bebelm_matvec", "bebelm_matmul", "bebelm_dequantize",
    "bebelm_attn_weights_create", "bebelm_attn_weights_destroy", "bebelm_attn_layer_step", "bebelm_attn_layer_batch",
    "bebelm_step_plan_create_layer", "bebelm_step_plan_launch_layer", "bebelm_head_create", "bebelm_head_destroy",
    "bebelm_head_logits", "bebelm_sample_greedy", "bebelm_gguf_open", "bebelm_gguf_from_bytes", "bebelm_gguf_close",
    "bebelm_gguf_header", "bebelm_gguf_tensor_at", "bebelm_gguf_find_tensor", "bebelm_gguf_key_at",
    "bebelm_gguf_get_u32", "bebelm_gguf_get_f32", "bebelm_gguf_get_str", "bebelm_gguf_get_u32_array",
    "bebelm_gguf_array_len", "bebelm_gguf_get_str_at", "bebelm_gguf_validate", "bebelm_attn_weights_from_gguf",
    "bebelm_head_from_gguf", "bebelm_step_plan_launch_allgather", "bebelm_attn_prefill_allgather",
]
GGML_F32, GGML_F16, GGML_Q4_K, GGML_Q6_K = 0, 1, 12, 14
IPC_HANDLE_BYTES = 64


class GgufTensor(C.Structure):
    """bebelm_gguf_tensor: one entry of the tensor table (TensorInfo, src/gguf.rs:120-139)."""
    _fields_ = [("name", C.c_void_p), ("name_len", C.c_size_t), ("n_dims", C.c_uint32), ("dims", C.c_uint64 * 8),
                ("n_elements", C.c_uint64), ("ggml_type", C.c_int), ("offset", C.c_uint64),
                ("data_start", C.c_uint64), ("data_len", C.c_uint64), ("data", C.c_void_p)]


class BebelmError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code


_lib = None


def load_library(path: str = LIB_PATH):
    """Loads the CUDA library (building it first if it is missing and nvcc exists)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        from . import build as _b
        _b.build()
    L = C.CDLL(path)
    vp, sz, i, f = C.c_void_p, C.c_size_t, C.c_int, C.c_float
    sig = {
        "bebelm_abi_version": ([], i),
        "bebelm_last_error": ([C.c_char_p, sz], i),
        "bebelm_device_count": ([C.POINTER(i)], i),
        "bebelm_attn_decode_host": ([vp, vp, vp, sz, i, i, i, vp], i),
        "bebelm_norm_rope_heads": ([vp, sz, i, i, vp, sz, f, f, i, vp], i),
        "bebelm_kv_pool_create": ([i, i, i, sz, i, i, i, C.POINTER(vp)], i),
        "bebelm_kv_pool_destroy": ([vp], i),
        "bebelm_kv_pool_free_pages": ([vp, C.POINTER(sz)], i),
        "bebelm_kv_create": ([i, i, i, sz, i, i, i, C.POINTER(vp)], i),
        "bebelm_kv_create_in_pool": ([vp, sz, C.POINTER(vp)], i),
        "bebelm_kv_destroy": ([vp], i),
        "bebelm_kv_clone": ([vp, C.POINTER(vp)], i),
        "bebelm_kv_clear": ([vp], i),
        "bebelm_kv_len": ([vp, C.POINTER(sz)], i),
        "bebelm_kv_layer_len": ([vp, i, C.POINTER(sz)], i),
        "bebelm_kv_pos": ([vp, C.POINTER(sz)], i),
        "bebelm_kv_set_pos": ([vp, sz], i),
        "bebelm_kv_evict_front": ([vp, sz], i),
        "bebelm_kv_append": ([vp, i, vp, vp, sz, i, vp], i),
        "bebelm_kv_read": ([vp, i, vp, vp, i, vp], i),
        "bebelm_attn_step": ([vp, i, i, vp, vp, vp, vp, vp, f, f, sz, vp, i, vp], i),
        "bebelm_attn_decode_cached": ([vp, i, i, vp, vp, i, vp], i),
        "bebelm_attn_decode_cached_noalloc": ([vp, i, i, vp, vp, vp], i),
        "bebelm_attn_prefill": ([vp, i, i, vp, vp, vp, i, sz, sz, vp, vp, f, f, vp, i, vp], i),
        "bebelm_attn_decode_batched": ([vp, i, i, i, vp, vp, vp, vp, vp, f, f, vp, vp, i, vp], i),
        "bebelm_kv_check": ([vp, vp], i),
        "bebelm_debug_expire_next_wait": ([i], i),
        "bebelm_peer_group_create": ([i, i, i, sz, vp, C.POINTER(vp)], i),
        "bebelm_peer_group_connect": ([vp, vp], i),
        "bebelm_peer_group_destroy": ([vp], i),
        "bebelm_attn_step_allgather": ([vp, vp, i, i, vp, vp, vp, vp, vp, f, f, sz, vp, i, vp], i),
        "bebelm_step_plan_create": ([vp, i, i, sz, C.POINTER(vp)], i),
        "bebelm_step_plan_launch": ([vp, vp, vp, vp, vp, vp, f, f, vp, vp], i),
        "bebelm_step_plan_launch_allgather": ([vp, vp, vp, vp, vp, vp, vp, f, f, vp, vp], i),
        "bebelm_attn_prefill_allgather": ([vp, vp, i, i, vp, vp, vp, i, sz, sz, vp, vp, f, f, vp, vp], i),
        "bebelm_step_plan_steps": ([vp, C.POINTER(C.c_ulonglong), vp], i),
        "bebelm_step_plan_finish": ([vp, vp], i),
        "bebelm_matvec": ([i, vp, sz, sz, vp, vp, i, vp], i),
        "bebelm_matmul": ([i, vp, sz, sz, vp, sz, vp, i, vp], i),
        "bebelm_dequantize": ([i, vp, sz, vp, i, vp], i),
        "bebelm_attn_weights_create": ([i, i, i, sz, i, vp, i, vp, i, vp, i, vp, vp, vp, C.POINTER(vp)], i),
        "bebelm_attn_weights_destroy": ([vp], i),
        "bebelm_attn_layer_step": ([vp, i, vp, vp, sz, f, f, vp, i, vp], i),
        "bebelm_attn_layer_batch": ([vp, i, vp, vp, sz, sz, i, f, f, vp, i, vp], i),
        "bebelm_step_plan_create_layer": ([vp, i, vp, sz, C.POINTER(vp)], i),
        "bebelm_step_plan_launch_layer": ([vp, vp, f, f, vp, vp], i),
        "bebelm_head_create": ([i, i, vp, sz, sz, vp, C.POINTER(vp)], i),
        "bebelm_head_destroy": ([vp], i),
        "bebelm_head_logits": ([vp, vp, f, vp, vp, i, vp], i),
        "bebelm_sample_greedy": ([vp, sz, vp, sz, f, vp, i, vp], i),
        "bebelm_gguf_open": ([C.c_char_p, C.POINTER(vp)], i),
        "bebelm_gguf_from_bytes": ([vp, sz, C.POINTER(vp)], i),
        "bebelm_gguf_close": ([vp], i),
        "bebelm_gguf_header": ([vp, C.POINTER(C.c_uint32), C.POINTER(C.c_uint64), C.POINTER(C.c_uint64),
                                C.POINTER(sz), C.POINTER(sz)], i),
        "bebelm_gguf_tensor_at": ([vp, sz, C.POINTER(GgufTensor)], i),
        "bebelm_gguf_find_tensor": ([vp, C.c_char_p, C.POINTER(GgufTensor)], i),
        "bebelm_gguf_key_at": ([vp, sz, C.POINTER(C.c_void_p), C.POINTER(sz), C.POINTER(i)], i),
        "bebelm_gguf_get_u32": ([vp, C.c_char_p, C.POINTER(C.c_uint32)], i),
        "bebelm_gguf_get_f32": ([vp, C.c_char_p, C.POINTER(f)], i),
        "bebelm_gguf_get_str": ([vp, C.c_char_p, C.c_char_p, sz, C.POINTER(sz)], i),
        "bebelm_gguf_get_u32_array": ([vp, C.c_char_p, C.POINTER(C.c_uint32), sz, C.POINTER(sz)], i),
        "bebelm_gguf_array_len": ([vp, C.c_char_p, C.POINTER(i), C.POINTER(sz)], i),
        "bebelm_gguf_get_str_at": ([vp, C.c_char_p, sz, C.POINTER(C.c_void_p), C.POINTER(sz)], i),
        "bebelm_gguf_validate": ([vp], i),
        "bebelm_attn_weights_from_gguf": ([vp, i, i, C.POINTER(vp)], i),
        "bebelm_head_from_gguf": ([vp, i, C.POINTER(vp)], i),
    }
    for name, (args, res) in sig.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = res
    _lib = L
    return L


def last_error() -> str:
    buf = C.create_string_buffer(1024)
    load_library().bebelm_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def _check(rc: int):
    if rc != 0:
        raise BebelmError(rc, last_error())


def device_count() -> int:
    n = C.c_int(0)
    _check(load_library().bebelm_device_count(C.byref(n)))
    return n.value


# ------------------------------------------------------------ buffer helpers --
def _is_torch(x) -> bool:
    return type(x).__module__.startswith("torch")


def _buf(x, dtype=np.float32):
    """Returns (pointer, mem kind, keepalive) for a numpy array or a CUDA tensor."""
    if _is_torch(x):
        if not x.is_cuda:
            x = x.detach().contiguous().numpy()
        else:
            if not x.is_contiguous():
                raise ValueError("device tensors must be contiguous")
            return x.data_ptr(), MEM_DEVICE, x
    a = np.ascontiguousarray(x, dtype=dtype)
    return a.ctypes.data, MEM_HOST, a


def _bufs(*xs, dtype=np.float32):
    out = [_buf(x, dtype) for x in xs]
    kinds = {m for _, m, _ in out}
    if len(kinds) != 1:
        raise ValueError("mix of host and device buffers in one call")
    return out, kinds.pop()


_torch = None


def _stream_ptr(stream, mem=MEM_DEVICE):
    """The cudaStream_t for a call. Host-memory calls synchronise before returning, so they
    run on the legacy default stream (NULL) unless one is given; device-memory calls default
    to torch's current stream."""
    global _torch
    if stream is None:
        if mem == MEM_HOST:
            return None
        if _torch is None:
            try:
                import torch
                _torch = torch if torch.cuda.is_available() else False
            except Exception:
                _torch = False
        return C.c_void_p(_torch.cuda.current_stream().cuda_stream) if _torch else None
    if hasattr(stream, "cuda_stream"):
        return C.c_void_p(stream.cuda_stream)
    return C.c_void_p(int(stream))


# ------------------------------------------------------------------ drop-ins --
def attention_decode(q, k, v, n_ctx: int, n_heads: int, n_kv_heads: int, head_dim: int) -> np.ndarray:
    """``attention_decode`` (src/kernels/attention.rs:17-26) on the GPU; host float32 in/out."""
    q = np.ascontiguousarray(q, np.float32).reshape(-1)
    k = np.ascontiguousarray(k, np.float32).reshape(-1)
    v = np.ascontiguousarray(v, np.float32).reshape(-1)
    if q.size != n_heads * head_dim or k.size != n_ctx * n_kv_heads * head_dim or v.size != k.size:
        raise ValueError("attention_decode: buffer sizes do not match the geometry")
    out = np.zeros(n_heads * head_dim, np.float32)
    kp = k.ctypes.data if k.size else None
    vp = v.ctypes.data if v.size else None
    _check(load_library().bebelm_attn_decode_host(q.ctypes.data, kp, vp, n_ctx, n_heads, n_kv_heads, head_dim,
                                                   out.ctypes.data))
    return out


def norm_rope_heads(buf, n_heads: int, head_dim: int, gain, pos: int, theta: float = ROPE_THETA,
                    eps: float = RMS_EPS, n_tokens: int = 1, stream=None):
    """``norm_rope_heads`` (src/model.rs:600-608) for n_tokens positions pos, pos+1, ...

    Host input: returns a new normed/roped float32 array. Device tensor: in place, returned."""
    if _is_torch(buf) and buf.is_cuda:
        (b, g), mem = _bufs(buf, gain)
        _check(load_library().bebelm_norm_rope_heads(b[0], n_tokens, n_heads, head_dim, g[0], pos, theta, eps, mem,
                                                      _stream_ptr(stream, mem)))
        return buf
    out = np.array(buf, np.float32, copy=True).reshape(-1)
    g = np.ascontiguousarray(gain, np.float32)
    _check(load_library().bebelm_norm_rope_heads(out.ctypes.data, n_tokens, n_heads, head_dim, g.ctypes.data, pos,
                                                  theta, eps, MEM_HOST, None))
    return out


# --------------------------------------------------------------------- cache --
class Pool:
    """A device page pool that several caches (sequences) draw from."""

    def __init__(self, n_layers: int, n_pages: int, n_kv_heads: int = N_KV_HEADS, head_dim: int = HEAD_DIM,
                 page_tokens: int = 64, device: int = 0, kv_dtype: int = F32):
        self._h = C.c_void_p()
        self.n_layers, self.n_kv_heads = n_layers, n_kv_heads
        _check(load_library().bebelm_kv_pool_create(n_layers, n_kv_heads, head_dim, n_pages, page_tokens, kv_dtype,
                                                    device, C.byref(self._h)))

    def free_pages(self) -> int:
        n = C.c_size_t()
        _check(load_library().bebelm_kv_pool_free_pages(self._h, C.byref(n)))
        return n.value

    def close(self):
        if self._h:
            _check(load_library().bebelm_kv_pool_destroy(self._h))
            self._h = C.c_void_p()

    def __del__(self):
        try:
            if self._h:
                load_library().bebelm_kv_pool_destroy(self._h)
        except Exception:
            pass


class Cache:
    """Device replacement of ``Cache`` (src/cache.rs:9-49) for the attention layers.

    ``layer`` indexes the cache's own attention layers (0..n_layers-1); a model
    maps its absolute attention layers (2, 6, 10, 14, 18, 21) onto these."""

    def __init__(self, n_layers: int = len(ATTENTION_LAYERS), n_kv_heads: int = N_KV_HEADS,
                 max_context: int = 32768, head_dim: int = HEAD_DIM, device: int = 0, pool: Pool | None = None,
                 kv_dtype: int = F32, _handle=None):
        """kv_dtype F32 keeps the reference's fp32 history; BF16 halves the bytes every decode
        step reads (K/V rounded to bf16 when appended)."""
        self.n_layers = n_layers if pool is None else pool.n_layers
        self.n_kv_heads = n_kv_heads if pool is None else pool.n_kv_heads
        self.head_dim = head_dim
        self.max_context = max_context
        self.pool = pool
        self.kv_dtype = kv_dtype
        L = load_library()
        if _handle is not None:
            self._h = _handle
        else:
            self._h = C.c_void_p()
            if pool is None:
                _check(L.bebelm_kv_create(n_layers, n_kv_heads, head_dim, max_context, 64, kv_dtype, device,
                                          C.byref(self._h)))
            else:
                _check(L.bebelm_kv_create_in_pool(pool._h, max_context, C.byref(self._h)))

    # -- src/cache.rs API -------------------------------------------------
    def kv_len(self) -> int:
        n = C.c_size_t()
        _check(load_library().bebelm_kv_len(self._h, C.byref(n)))
        return n.value

    def layer_len(self, layer: int) -> int:
        n = C.c_size_t()
        _check(load_library().bebelm_kv_layer_len(self._h, layer, C.byref(n)))
        return n.value

    @property
    def pos(self) -> int:
        n = C.c_size_t()
        _check(load_library().bebelm_kv_pos(self._h, C.byref(n)))
        return n.value

    @pos.setter
    def pos(self, p: int):
        _check(load_library().bebelm_kv_set_pos(self._h, p))

    def evict_front(self, n: int) -> None:
        _check(load_library().bebelm_kv_evict_front(self._h, n))

    def clone(self) -> "Cache":
        h = C.c_void_p()
        _check(load_library().bebelm_kv_clone(self._h, C.byref(h)))
        return Cache(self.n_layers, self.n_kv_heads, self.max_context, self.head_dim, pool=self.pool,
                     kv_dtype=self.kv_dtype, _handle=h)

    def clear(self) -> None:
        _check(load_library().bebelm_kv_clear(self._h))

    def append(self, layer: int, k, v, stream=None) -> None:
        """``cache.k[layer].extend_from_slice(k)`` and the same for v."""
        (kb, vb), mem = _bufs(k, v)
        t = (kb[2].size if mem == MEM_HOST else kb[2].numel()) // (self.n_kv_heads * self.head_dim)
        _check(load_library().bebelm_kv_append(self._h, layer, kb[0], vb[0], t, mem, _stream_ptr(stream, mem)))

    def read(self, layer: int):
        """The window of one layer as host arrays (k, v), each [len, n_kv*64] — what
        ``cache.k[layer]`` / ``cache.v[layer]`` hold in the reference."""
        n = self.layer_len(layer)
        k = np.zeros((n, self.n_kv_heads * self.head_dim), np.float32)
        v = np.zeros_like(k)
        if n:
            _check(load_library().bebelm_kv_read(self._h, layer, k.ctypes.data, v.ctypes.data, MEM_HOST, None))
        return k, v

    # -- fused ops ----------------------------------------------------------
    def attn_step(self, layer: int, q, k, v, q_gain, k_gain, pos: int, theta: float = ROPE_THETA,
                  eps: float = RMS_EPS, out=None, stream=None):
        """src/model.rs:440-451 (norm+RoPE, append, decode). Returns out [n_heads*64]."""
        (qb, kb, vb, qg, kg), mem = _bufs(q, k, v, q_gain, k_gain)
        n_heads = (qb[2].size if mem == MEM_HOST else qb[2].numel()) // self.head_dim
        if out is None:
            out = np.zeros(n_heads * self.head_dim, np.float32) if mem == MEM_HOST else qb[2].new_empty(
                n_heads * self.head_dim, dtype=qb[2].dtype)
        ob, _, _ = _buf(out)
        _check(load_library().bebelm_attn_step(self._h, layer, n_heads, qb[0], kb[0], vb[0], qg[0], kg[0], theta, eps,
                                               pos, ob, mem, _stream_ptr(stream, mem)))
        return out

    def attn_step_allgather(self, group: "PeerGroup", layer: int, q, k, v, q_gain, k_gain, pos: int,
                            theta: float = ROPE_THETA, eps: float = RMS_EPS, out=None, stream=None):
        """:meth:`attn_step` on this rank's heads with the all-gather fused into the decode
        kernel (peer stores over NVLink). q/k/v are this rank's slices; returns the full
        [world * n_heads * 64] output in rank order."""
        (qb, kb, vb, qg, kg), mem = _bufs(q, k, v, q_gain, k_gain)
        n_heads = (qb[2].size if mem == MEM_HOST else qb[2].numel()) // self.head_dim
        n_out = group.world * n_heads * self.head_dim
        if out is None:
            out = np.zeros(n_out, np.float32) if mem == MEM_HOST else qb[2].new_empty(n_out, dtype=qb[2].dtype)
        ob, _, _ = _buf(out)
        _check(load_library().bebelm_attn_step_allgather(self._h, group._h, layer, n_heads, qb[0], kb[0], vb[0], qg[0],
                                                         kg[0], theta, eps, pos, ob, mem, _stream_ptr(stream, mem)))
        return out

    def attn_prefill_allgather(self, group: "PeerGroup", layer: int, q, k, v, q_gain, k_gain, pos0: int,
                               theta: float = ROPE_THETA, eps: float = RMS_EPS, out=None, stream=None,
                               n_heads: int | None = None):
        """:meth:`attn_prefill` on this rank's heads of the full rows q [t, world*n_heads*64],
        k/v [t, world*n_kv*64] (CUDA tensors, bf16, or float32 for the tensor cores), gathered
        over ``group``: returns out [t, world*n_heads*64] float32."""
        import torch
        world = group.world
        if n_heads is None:
            n_heads = q.shape[-1] // (self.head_dim * world)
        t = q.numel() // (world * n_heads * self.head_dim)
        in_dtype = BF16 if q.dtype == torch.bfloat16 else F32_TENSOR
        if out is None:
            out = torch.empty((t, world * n_heads * self.head_dim), dtype=torch.float32, device=q.device)
        _check(load_library().bebelm_attn_prefill_allgather(
            self._h, group._h, layer, n_heads, q.data_ptr(), k.data_ptr(), v.data_ptr(), in_dtype, t, pos0,
            q_gain.data_ptr(), k_gain.data_ptr(), theta, eps, out.data_ptr(), _stream_ptr(stream)))
        return out

    def check(self, stream=None) -> None:
        """Synchronises and raises if a bounded device-side wait gave up (device-memory calls)."""
        _check(load_library().bebelm_kv_check(self._h, _stream_ptr(stream)))

    def step_plan(self, layer: int, n_heads: int = N_HEADS, window: int = 0) -> "StepPlan":
        """A device-driven decode step for ``layer`` (see :class:`StepPlan`)."""
        return StepPlan(self, layer, n_heads, window)

    def decode(self, layer: int, q, out=None, stream=None):
        """``attention_decode`` over the cached window of ``layer`` (no append); q normed+roped."""
        (qb,), mem = _bufs(q)
        n_heads = (qb[2].size if mem == MEM_HOST else qb[2].numel()) // self.head_dim
        if out is None:
            out = np.zeros(n_heads * self.head_dim, np.float32) if mem == MEM_HOST else qb[2].new_empty(
                n_heads * self.head_dim)
        ob, _, _ = _buf(out)
        _check(load_library().bebelm_attn_decode_cached(self._h, layer, n_heads, qb[0], ob, mem, _stream_ptr(stream, mem)))
        return out

    def attn_prefill(self, layer: int, q, k, v, q_gain, k_gain, pos0: int, theta: float = ROPE_THETA,
                     eps: float = RMS_EPS, out=None, stream=None, n_heads: int = N_HEADS,
                     tensor_cores: bool = False):
        """src/model.rs:232-254 for t tokens. q [t, n_heads*64], k/v [t, n_kv*64] (float32 or bf16
        tensors). Returns out [t, n_heads*64] float32. bf16 inputs always take the tensor cores;
        float32 inputs take them when ``tensor_cores`` is set (else the reference's fp32 arithmetic)."""
        is_dev = _is_torch(q) and q.is_cuda
        if is_dev:
            import torch
            in_dtype = BF16 if q.dtype == torch.bfloat16 else (F32_TENSOR if tensor_cores else F32)
            t = q.numel() // (n_heads * self.head_dim)
            if out is None:
                out = torch.empty((t, n_heads * self.head_dim), dtype=torch.float32, device=q.device)
            ptrs = [C.c_void_p(x.data_ptr()) for x in (q, k, v, q_gain, k_gain, out)]
            mem = MEM_DEVICE
            keep = (q, k, v, q_gain, k_gain, out)
        else:
            q = np.ascontiguousarray(q)
            in_dtype = F32_TENSOR if tensor_cores else F32
            if q.dtype != np.float32:
                q = q.astype(np.float32)
            k = np.ascontiguousarray(k, np.float32)
            v = np.ascontiguousarray(v, np.float32)
            qg = np.ascontiguousarray(q_gain, np.float32)
            kg = np.ascontiguousarray(k_gain, np.float32)
            t = q.size // (n_heads * self.head_dim)
            if out is None:
                out = np.zeros((t, n_heads * self.head_dim), np.float32)
            elif not (isinstance(out, np.ndarray) and out.dtype == np.float32 and out.flags.c_contiguous
                      and out.size == t * n_heads * self.head_dim):
                raise ValueError("out must be a C-contiguous float32 array of t * n_heads * 64 elements")
            keep = (q, k, v, qg, kg, out)
            ptrs = [C.c_void_p(x.ctypes.data) for x in keep]
            mem = MEM_HOST
        _check(load_library().bebelm_attn_prefill(self._h, layer, n_heads, ptrs[0], ptrs[1], ptrs[2], in_dtype, t,
                                                  pos0, ptrs[3], ptrs[4], theta, eps, ptrs[5], mem,
                                                  _stream_ptr(stream, mem)))
        del keep
        return out

    def close(self):
        if self._h:
            _check(load_library().bebelm_kv_destroy(self._h))
            self._h = C.c_void_p()

    def __del__(self):
        try:
            if self._h:
                load_library().bebelm_kv_destroy(self._h)
        except Exception:
            pass


def _raw(x):
    """(pointer, mem, keepalive) for raw weight bytes: a uint8 numpy array / bytes, or a CUDA tensor."""
    if _is_torch(x):
        if not x.is_cuda:
            x = x.detach().contiguous().numpy()
        else:
            return x.data_ptr(), MEM_DEVICE, x
    a = np.ascontiguousarray(np.frombuffer(x, np.uint8) if isinstance(x, (bytes, bytearray)) else x).view(np.uint8)
    return a.ctypes.data, MEM_HOST, a


def matmul(dtype: int, w, n_in: int, n_out: int, x, n_tokens: int = 1, out=None, stream=None):
    """``matmul`` / ``matvec`` (src/kernels/matmul.rs:850-1013) on the GPU: y [n_tokens, n_out] = W x.
    w: the packed weight bytes (numpy uint8 / bytes, or a CUDA uint8 tensor); x float32 [n_tokens, n_in]."""
    wp, wm, wk = _raw(w)
    xb, xm, xk = _buf(x)
    if wm != xm:
        raise ValueError("weights and activations must both be host or both be device buffers")
    if out is None:
        out = np.zeros((n_tokens, n_out), np.float32) if xm == MEM_HOST else xk.new_empty((n_tokens, n_out))
    ob, _, _ = _buf(out)
    _check(load_library().bebelm_matmul(dtype, wp, n_in, n_out, xb, n_tokens, ob, xm, _stream_ptr(stream, xm)))
    return out.reshape(-1) if n_tokens == 1 and out.ndim > 1 and xm == MEM_HOST else out


def matvec(dtype: int, w, n_in: int, n_out: int, x, out=None, stream=None):
    return matmul(dtype, w, n_in, n_out, x, 1, out=out, stream=stream)


def dequantize(dtype: int, data, n: int, stream=None) -> np.ndarray:
    """``dequantize`` (src/kernels/dequant.rs:151-186) on the GPU; host bytes in, float32 out."""
    dp, dm, dk = _raw(data)
    if dm != MEM_HOST:
        raise ValueError("dequantize takes host bytes")
    out = np.zeros(n, np.float32)
    _check(load_library().bebelm_dequantize(dtype, dp, n, out.ctypes.data, MEM_HOST, None))
    return out


class AttnWeights:
    """A layer's attention weights on the device: GGUF tensors as stored (packed bytes + ggml
    dtype) for attn_q / attn_k / attn_v / attn_output, and the q/k norm gains."""

    def __init__(self, wq, wk, wv, wo, q_gain, k_gain, n_heads: int = N_HEADS, n_kv_heads: int = N_KV_HEADS,
                 hidden: int = HIDDEN, device: int = 0):
        """wq/wk/wv/wo: (dtype, bytes) pairs (bytes: numpy uint8 or bytes)."""
        self.n_heads, self.n_kv, self.hidden = n_heads, n_kv_heads, hidden
        keep = [np.ascontiguousarray(np.frombuffer(b, np.uint8) if isinstance(b, (bytes, bytearray)) else b).view(np.uint8)
                for _, b in (wq, wk, wv, wo)]
        g = [np.ascontiguousarray(x, np.float32) for x in (q_gain, k_gain)]
        self._h = C.c_void_p()
        _check(load_library().bebelm_attn_weights_create(
            device, n_heads, n_kv_heads, hidden, wq[0], keep[0].ctypes.data, wk[0], keep[1].ctypes.data, wv[0],
            keep[2].ctypes.data, wo[0], keep[3].ctypes.data, g[0].ctypes.data, g[1].ctypes.data, C.byref(self._h)))

    def close(self):
        if self._h:
            load_library().bebelm_attn_weights_destroy(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Head:
    """The logits head on the device (``logits_from_hidden``, src/model.rs:379-388): the final
    RMSNorm (``token_embd_norm``) and the tied ``token_embd`` matvec, as stored (ggml dtype,
    [vocab][hidden] packed bytes), plus the greedy token."""

    def __init__(self, dtype: int, token_embd, hidden: int, vocab: int, norm_gain, device: int = 0):
        w = np.ascontiguousarray(np.frombuffer(token_embd, np.uint8) if isinstance(token_embd, (bytes, bytearray))
                                 else token_embd).view(np.uint8)
        g = np.ascontiguousarray(norm_gain, np.float32)
        self.hidden, self.vocab = hidden, vocab
        self._h = C.c_void_p()
        _check(load_library().bebelm_head_create(device, dtype, w.ctypes.data, hidden, vocab, g.ctypes.data,
                                                 C.byref(self._h)))

    def logits(self, h, eps: float = RMS_EPS, logits=True, token=True, stream=None):
        """h [hidden] -> (logits [vocab] or None, token or None). Host arrays give numpy results
        (token an int); device tensors give device results (token an int32 tensor [1]) computed
        without leaving the device."""
        (hb,), mem = _bufs(h)
        if mem == MEM_HOST:
            lg = np.zeros(self.vocab, np.float32) if logits else None
            tk = np.zeros(1, np.uint32) if token else None
        else:
            import torch
            lg = hb[2].new_empty(self.vocab) if logits else None
            tk = hb[2].new_zeros(1, dtype=torch.int32) if token else None
        lp = _buf(lg)[0] if lg is not None else None
        tp = None if tk is None else (tk.ctypes.data if mem == MEM_HOST else tk.data_ptr())
        _check(load_library().bebelm_head_logits(self._h, hb[0], eps, lp, tp, mem, _stream_ptr(stream, mem)))
        if mem == MEM_HOST and tk is not None:
            tk = int(tk[0])
        return lg, tk

    def close(self):
        if self._h:
            load_library().bebelm_head_destroy(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def sample_greedy(logits, history=(), repeat_penalty: float = 1.0, stream=None):
    """``Sampler::sample`` with temperature <= 0 (src/sampler.rs:64-88): presence penalty on
    ``logits`` in place, then ``argmax``. Host: returns the token id; device (CUDA float32
    tensor logits, history a CUDA int32 tensor or empty): returns an int32 tensor [1]."""
    (lb,), mem = _bufs(logits)
    n = lb[2].size if mem == MEM_HOST else lb[2].numel()
    if mem == MEM_HOST:
        hist = np.ascontiguousarray(np.asarray(history, np.uint32))
        tok = np.zeros(1, np.uint32)
        _check(load_library().bebelm_sample_greedy(lb[0], n, hist.ctypes.data if hist.size else None, hist.size,
                                                   repeat_penalty, tok.ctypes.data, mem, None))
        return int(tok[0])
    import torch
    hist = history if hasattr(history, "data_ptr") else torch.tensor(list(history), dtype=torch.int32,
                                                                      device=lb[2].device)
    tok = torch.zeros(1, dtype=torch.int32, device=lb[2].device)
    _check(load_library().bebelm_sample_greedy(lb[0], n, hist.data_ptr() if hist.numel() else None, hist.numel(),
                                               repeat_penalty, tok.data_ptr(), mem, _stream_ptr(stream, mem)))
    return tok


def attn_layer_step(cache: "Cache", layer: int, weights: AttnWeights, x, pos: int, theta: float = ROPE_THETA,
                    eps: float = RMS_EPS, out=None, stream=None):
    """``attn_step`` (src/model.rs:430-455) whole: x [hidden] -> out [hidden]."""
    (xb,), mem = _bufs(x)
    if out is None:
        out = np.zeros(weights.hidden, np.float32) if mem == MEM_HOST else xb[2].new_empty(weights.hidden)
    ob, _, _ = _buf(out)
    _check(load_library().bebelm_attn_layer_step(cache._h, layer, weights._h, xb[0], pos, theta, eps, ob, mem,
                                                 _stream_ptr(stream, mem)))
    return out


def attn_layer_batch(cache: "Cache", layer: int, weights: AttnWeights, x, pos0: int, tensor_cores: bool = True,
                     theta: float = ROPE_THETA, eps: float = RMS_EPS, out=None, stream=None):
    """``attn_batch`` (src/model.rs:224-258) whole: x [t, hidden] -> out [t, hidden]."""
    (xb,), mem = _bufs(x)
    n = xb[2].size if mem == MEM_HOST else xb[2].numel()
    t = n // weights.hidden
    if out is None:
        out = np.zeros((t, weights.hidden), np.float32) if mem == MEM_HOST else xb[2].new_empty((t, weights.hidden))
    ob, _, _ = _buf(out)
    _check(load_library().bebelm_attn_layer_batch(cache._h, layer, weights._h, xb[0], t, pos0, 1 if tensor_cores else 0,
                                                  theta, eps, ob, mem, _stream_ptr(stream, mem)))
    return out


class StepPlan:
    """Device-driven decode steps of one cache layer, for CUDA-graph capture.

    Each :meth:`launch` is the ``attn_step`` of the next token (position ``cache.pos + n`` for
    the n-th launch), with the window sliding once it holds ``window`` positions; the launch
    does no host work that depends on the step, so ``torch.cuda.graph`` can capture it and
    replays advance the sequence. Device tensors only. :meth:`finish` writes the steps back
    into the cache; until then other calls on the cache are refused."""

    def __init__(self, cache: "Cache", layer: int, n_heads: int = N_HEADS, window: int = 0,
                 weights: "AttnWeights | None" = None):
        """With ``weights`` the plan is the whole operator (:meth:`launch_layer`)."""
        self.cache, self.layer, self.n_heads, self.weights = cache, layer, n_heads, weights
        self._h = C.c_void_p()
        if weights is None:
            _check(load_library().bebelm_step_plan_create(cache._h, layer, n_heads, window, C.byref(self._h)))
        else:
            _check(load_library().bebelm_step_plan_create_layer(cache._h, layer, weights._h, window,
                                                                C.byref(self._h)))

    def launch_layer(self, x, out, theta: float = ROPE_THETA, eps: float = RMS_EPS, stream=None):
        """One token through the whole operator: x [hidden] -> out [hidden] (CUDA tensors)."""
        for t in (x, out):
            if not (_is_torch(t) and t.is_cuda and t.is_contiguous()):
                raise ValueError("step plans take contiguous CUDA tensors")
        _check(load_library().bebelm_step_plan_launch_layer(self._h, x.data_ptr(), theta, eps, out.data_ptr(),
                                                            _stream_ptr(stream)))
        return out

    def launch(self, q, k, v, q_gain, k_gain, out, theta: float = ROPE_THETA, eps: float = RMS_EPS, stream=None):
        for x in (q, k, v, q_gain, k_gain, out):
            if not (_is_torch(x) and x.is_cuda and x.is_contiguous()):
                raise ValueError("step plans take contiguous CUDA tensors")
        _check(load_library().bebelm_step_plan_launch(self._h, q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                                      q_gain.data_ptr(), k_gain.data_ptr(), theta, eps,
                                                      out.data_ptr(), _stream_ptr(stream)))
        return out

    def launch_allgather(self, group: "PeerGroup", q, k, v, q_gain, k_gain, out, theta: float = ROPE_THETA,
                         eps: float = RMS_EPS, stream=None):
        """:meth:`launch` on this rank's heads, gathered over ``group`` into out [world*n_heads*64];
        capturable in a CUDA graph on every rank."""
        for x in (q, k, v, q_gain, k_gain, out):
            if not (_is_torch(x) and x.is_cuda and x.is_contiguous()):
                raise ValueError("step plans take contiguous CUDA tensors")
        _check(load_library().bebelm_step_plan_launch_allgather(
            self._h, group._h, q.data_ptr(), k.data_ptr(), v.data_ptr(), q_gain.data_ptr(), k_gain.data_ptr(), theta,
            eps, out.data_ptr(), _stream_ptr(stream)))
        return out

    def steps(self, stream=None) -> int:
        n = C.c_ulonglong()
        _check(load_library().bebelm_step_plan_steps(self._h, C.byref(n), _stream_ptr(stream)))
        return n.value

    def finish(self, stream=None) -> None:
        if self._h:
            h, self._h = self._h, C.c_void_p()
            _check(load_library().bebelm_step_plan_finish(h, _stream_ptr(stream)))


class PeerGroup:
    """Landing zones for the fused decode + all-gather of KV-head sharding (one per rank).

    Collective protocol: construct on every rank, exchange :attr:`handle` (bytes), then call
    :meth:`connect` with all ranks' handles in rank order. ``slice_floats`` = n_heads*64 of
    one rank. Close collectively (host barrier first)."""

    def __init__(self, world: int, rank: int, slice_floats: int, device: int = 0):
        self.world, self.rank, self.slice = world, rank, slice_floats
        self._h = C.c_void_p()
        buf = C.create_string_buffer(IPC_HANDLE_BYTES)
        _check(load_library().bebelm_peer_group_create(device, world, rank, slice_floats, buf, C.byref(self._h)))
        self.handle = buf.raw

    def connect(self, handles) -> None:
        if len(handles) != self.world or any(len(h) != IPC_HANDLE_BYTES for h in handles):
            raise ValueError(f"need {self.world} handles of {IPC_HANDLE_BYTES} bytes")
        blob = C.create_string_buffer(b"".join(handles), IPC_HANDLE_BYTES * self.world)
        _check(load_library().bebelm_peer_group_connect(self._h, blob))

    def close(self) -> None:
        if self._h:
            load_library().bebelm_peer_group_destroy(self._h)
            self._h = C.c_void_p()


def attn_decode_batched(caches, layer: int, q, k, v, q_gain, k_gain, pos, theta: float = ROPE_THETA,
                        eps: float = RMS_EPS, out=None, stream=None):
    """One decode token for each cache (all in one :class:`Pool`): q [n, n_heads*64],
    k/v [n, n_kv*64]. Returns out [n, n_heads*64]."""
    n = len(caches)
    arr = (C.c_void_p * n)(*[c._h for c in caches])
    (qb, kb, vb, qg, kg), mem = _bufs(q, k, v, q_gain, k_gain)
    numel = qb[2].size if mem == MEM_HOST else qb[2].numel()
    n_heads = numel // (n * caches[0].head_dim)
    if out is None:
        out = np.zeros((n, n_heads * 64), np.float32) if mem == MEM_HOST else qb[2].new_empty((n, n_heads * 64))
    ob, _, _ = _buf(out)
    posa = (C.c_size_t * n)(*[int(p) for p in pos])
    _check(load_library().bebelm_attn_decode_batched(arr, n, layer, n_heads, qb[0], kb[0], vb[0], qg[0], kg[0], theta,
                                                     eps, posa, ob, mem, _stream_ptr(stream, mem)))
    return out


# ------------------------------------------------------------------ GGUF --
class Gguf:
    """``GgufFile`` (src/gguf.rs:157-298) over the library's native reader: ``Gguf(path)``
    memory-maps a file (GgufFile::open), ``Gguf(data=bytes)`` parses a copy of a buffer
    (GgufFile::from_bytes). Raises :class:`BebelmError` (ERR_FORMAT with the reference's
    wording) on a malformed file."""

    def __init__(self, path: str | None = None, data: bytes | None = None):
        L = load_library()
        self._h = C.c_void_p()
        if path is not None:
            _check(L.bebelm_gguf_open(os.fsencode(path), C.byref(self._h)))
        else:
            buf = C.create_string_buffer(bytes(data), len(data)) if data else None
            _check(L.bebelm_gguf_from_bytes(buf, len(data or b""), C.byref(self._h)))
        ver, al, off = C.c_uint32(), C.c_uint64(), C.c_uint64()
        nt, nk = C.c_size_t(), C.c_size_t()
        _check(L.bebelm_gguf_header(self._h, C.byref(ver), C.byref(al), C.byref(off), C.byref(nt), C.byref(nk)))
        self.version, self.alignment, self.data_offset = ver.value, al.value, off.value
        self.n_tensors, self.n_kv = nt.value, nk.value

    @staticmethod
    def _info(t: GgufTensor) -> dict:
        return {"name": C.string_at(t.name, t.name_len).decode(), "dims": [t.dims[d] for d in range(min(t.n_dims, 8))],
                "n_dims": t.n_dims, "ggml_type": t.ggml_type, "n_elements": t.n_elements, "offset": t.offset,
                "data_start": t.data_start, "data_len": t.data_len, "data_ptr": t.data}

    @property
    def tensors(self) -> list:
        out = []
        for i in range(self.n_tensors):
            t = GgufTensor()
            _check(load_library().bebelm_gguf_tensor_at(self._h, i, C.byref(t)))
            out.append(self._info(t))
        return out

    def tensor(self, name: str) -> dict | None:
        t = GgufTensor()
        rc = load_library().bebelm_gguf_find_tensor(self._h, name.encode(), C.byref(t))
        if rc == ERR_NOT_FOUND:
            return None
        _check(rc)
        return self._info(t)

    def tensor_data(self, name: str) -> bytes:
        t = self.tensor(name)
        return C.string_at(t["data_ptr"], t["data_len"])

    def keys(self) -> list:
        """[(key, value type)] in file order."""
        out = []
        for i in range(self.n_kv):
            k, n, vt = C.c_void_p(), C.c_size_t(), C.c_int()
            _check(load_library().bebelm_gguf_key_at(self._h, i, C.byref(k), C.byref(n), C.byref(vt)))
            out.append((C.string_at(k, n.value).decode(), vt.value))
        return out

    def get_u32(self, key: str):
        v = C.c_uint32()
        rc = load_library().bebelm_gguf_get_u32(self._h, key.encode(), C.byref(v))
        if rc == ERR_NOT_FOUND:
            return None
        _check(rc)
        return v.value

    def get_f32(self, key: str):
        v = C.c_float()
        rc = load_library().bebelm_gguf_get_f32(self._h, key.encode(), C.byref(v))
        if rc == ERR_NOT_FOUND:
            return None
        _check(rc)
        return v.value

    def get_str(self, key: str):
        n = C.c_size_t()
        L = load_library()
        rc = L.bebelm_gguf_get_str(self._h, key.encode(), None, 0, C.byref(n))
        if rc == ERR_NOT_FOUND:
            return None
        _check(rc)
        buf = C.create_string_buffer(n.value + 1)
        _check(L.bebelm_gguf_get_str(self._h, key.encode(), buf, n.value + 1, C.byref(n)))
        return buf.raw[: n.value].decode()

    def get_u32_array(self, key: str):
        n = C.c_size_t()
        L = load_library()
        rc = L.bebelm_gguf_get_u32_array(self._h, key.encode(), None, 0, C.byref(n))
        if rc == ERR_NOT_FOUND:
            return None
        _check(rc)
        out = (C.c_uint32 * max(n.value, 1))()
        _check(L.bebelm_gguf_get_u32_array(self._h, key.encode(), out, n.value, C.byref(n)))
        return list(out[: n.value])

    def get_str_array(self, key: str):
        et, n = C.c_int(), C.c_size_t()
        L = load_library()
        rc = L.bebelm_gguf_array_len(self._h, key.encode(), C.byref(et), C.byref(n))
        if rc == ERR_NOT_FOUND or et.value != 8:
            return None
        _check(rc)
        out = []
        for i in range(n.value):
            p, ln = C.c_void_p(), C.c_size_t()
            _check(L.bebelm_gguf_get_str_at(self._h, key.encode(), i, C.byref(p), C.byref(ln)))
            out.append(C.string_at(p, ln.value).decode())
        return out

    def architecture(self):
        return self.get_str("general.architecture")

    def validate(self) -> None:
        """config::validate (src/config.rs:50-96)."""
        _check(load_library().bebelm_gguf_validate(self._h))

    def attn_weights(self, block: int, device: int = 0) -> "AttnWeights":
        """The attention weights of model block ``block`` (blk.N.attn_*), uploaded to ``device``."""
        w = AttnWeights.__new__(AttnWeights)
        w._h = C.c_void_p()
        _check(load_library().bebelm_attn_weights_from_gguf(self._h, block, device, C.byref(w._h)))
        q, k = self.tensor(f"blk.{block}.attn_q.weight"), self.tensor(f"blk.{block}.attn_k.weight")
        w.hidden, w.n_heads, w.n_kv = q["dims"][0], q["dims"][1] // HEAD_DIM, k["dims"][1] // HEAD_DIM
        return w

    def head(self, device: int = 0) -> "Head":
        """The logits head (token_embd + token_embd_norm), uploaded to ``device``."""
        h = Head.__new__(Head)
        h._h = C.c_void_p()
        _check(load_library().bebelm_head_from_gguf(self._h, device, C.byref(h._h)))
        t = self.tensor("token_embd.weight")
        h.hidden, h.vocab = t["dims"][0], t["dims"][1]
        return h

    def close(self):
        if self._h:
            load_library().bebelm_gguf_close(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
