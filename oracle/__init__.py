"""CPU oracle for BebeLM's attention hot path — TEST INFRASTRUCTURE ONLY.

Loads ``oracle/liboracle.so`` (built from ``oracle/bebelm_oracle.c`` by
``oracle/Makefile``) and exposes the reference's arithmetic to numpy callers.
Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` may import this package; the product (``bebelm_b200``) never does.

``Cache`` restates ``src/cache.rs:9-49`` of the reference (per-layer growable
K/V histories, ``kv_len``, ``evict_front``, ``clone``) as the checker for the
device cache's window semantics.
"""
from __future__ import annotations

import copy
import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i64p = np.ctypeslib.ndpointer(np.int64, flags="C_CONTIGUOUS")


def build(force: bool = False) -> str:
    """Compile the C restatement (seconds). Returns the library path."""
    srcs = [os.path.join(_HERE, f) for f in ("bebelm_oracle.c", "quant_oracle.c")]
    if force or not os.path.exists(_LIB_PATH) or any(os.path.getmtime(_LIB_PATH) < os.path.getmtime(f) for f in srcs):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        L = C.CDLL(_LIB_PATH)
        sz = C.c_size_t
        L.orc_fill_normal.argtypes = [C.c_uint64, sz, C.c_float, C.c_float, _f32p]
        L.orc_fill_uniform_int.argtypes = [C.c_uint64, sz, C.c_int64, C.c_int64, _i64p]
        L.orc_dot.argtypes = [_f32p, _f32p, sz]
        L.orc_dot.restype = C.c_float
        L.orc_softmax.argtypes = [_f32p, sz]
        L.orc_rmsnorm.argtypes = [_f32p, _f32p, C.c_float, _f32p, sz]
        L.orc_rope_neox.argtypes = [_f32p, sz, sz, C.c_float]
        L.orc_norm_rope_heads.argtypes = [_f32p, C.c_int, C.c_int, _f32p, sz, C.c_float, C.c_float]
        L.orc_attention_decode.argtypes = [_f32p, _f32p, _f32p, sz, C.c_int, C.c_int, C.c_int, _f32p]
        L.orc_attention_decode_mt.argtypes = L.orc_attention_decode.argtypes + [C.c_int]
        L.orc_attn_batch.argtypes = [_f32p, _f32p, _f32p, sz, sz, _f32p, _f32p, C.c_float, C.c_float,
                                     C.c_int, C.c_int, C.c_int, _f32p, _f32p, C.POINTER(sz), _f32p, C.c_int]
        L.orc_attn_step.argtypes = [_f32p, _f32p, _f32p, sz, _f32p, _f32p, C.c_float, C.c_float,
                                    C.c_int, C.c_int, C.c_int, _f32p, _f32p, C.POINTER(sz), _f32p, C.c_int]
        L.orc_max_threads.restype = C.c_int
        u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
        i8p = np.ctypeslib.ndpointer(np.int8, flags="C_CONTIGUOUS")
        i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
        L.orc_f16_to_f32.argtypes = [C.c_uint16]
        L.orc_f16_to_f32.restype = C.c_float
        L.orc_dequantize.argtypes = [C.c_int, u8p, sz, _f32p]
        L.orc_quantize_q8.argtypes = [_f32p, sz, i8p, _f32p, i32p]
        L.orc_matvec.argtypes = [C.c_int, u8p, sz, sz, _f32p, _f32p, _f32p, i8p, _f32p, i32p]
        L.orc_matmul.argtypes = [C.c_int, u8p, sz, sz, _f32p, sz, _f32p, _f32p, i8p, _f32p, i32p]
        u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
        L.orc_argmax.argtypes = [_f32p, sz]
        L.orc_argmax.restype = sz
        L.orc_sample_greedy.argtypes = [_f32p, sz, u32p, sz, C.c_float, u32p]
        _lib = L
    return _lib


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


# ------------------------------------------------------------------ inputs --
def normal(seed: int, shape, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    """Seeded N(mean, std) float32 (SplitMix64 + Box-Muller, see bebelm_oracle.c)."""
    n = int(np.prod(shape))
    out = np.empty(max(n, 1), np.float32)
    lib().orc_fill_normal(seed, n, mean, std, out)
    return out[:n].reshape(shape)


def uniform_int(seed: int, n: int, lo: int, hi: int) -> np.ndarray:
    out = np.empty(max(n, 1), np.int64)
    lib().orc_fill_uniform_int(seed, n, lo, hi, out)
    return out[:n]


def max_threads() -> int:
    return lib().orc_max_threads()


# ------------------------------------------------------- elementary kernels --
def dot(a, b) -> float:
    a, b = _f32(a), _f32(b)
    if a.size == 0:
        return 0.0
    return float(lib().orc_dot(a, b, a.size))


def softmax(x) -> np.ndarray:
    x = _f32(x).copy()
    if x.size:
        lib().orc_softmax(x, x.size)
    return x


def rmsnorm(x, gain, eps: float) -> np.ndarray:
    x, g = _f32(x), _f32(gain)
    out = np.empty_like(x)
    lib().orc_rmsnorm(x, g, eps, out, x.size)
    return out


def rope_neox(x, pos: int, freq_base: float) -> np.ndarray:
    x = _f32(x).copy()
    lib().orc_rope_neox(x, x.size, pos, freq_base)
    return x


def norm_rope_heads(buf, n_heads: int, head_dim: int, gain, pos: int, theta: float,
                    eps: float = 1e-5) -> np.ndarray:
    b = _f32(buf).copy().reshape(-1)
    lib().orc_norm_rope_heads(b, n_heads, head_dim, _f32(gain), pos, theta, eps)
    return b


def attention_decode(q, k, v, n_ctx: int, n_heads: int, n_kv_heads: int, head_dim: int,
                     n_threads: int = 1) -> np.ndarray:
    q, k, v = _f32(q).reshape(-1), _f32(k).reshape(-1), _f32(v).reshape(-1)
    if k.size == 0:
        k = np.zeros(1, np.float32)
        v = np.zeros(1, np.float32)
    out = np.zeros(n_heads * head_dim, np.float32)
    if n_threads > 1:
        rc = lib().orc_attention_decode_mt(q, k, v, n_ctx, n_heads, n_kv_heads, head_dim, out, n_threads)
    else:
        rc = lib().orc_attention_decode(q, k, v, n_ctx, n_heads, n_kv_heads, head_dim, out)
    if rc:
        raise ValueError(f"oracle attention_decode failed: {rc}")
    return out


def attn_batch(q, k, v, pos0: int, q_gain, k_gain, theta: float, eps: float, n_heads: int,
               n_kv_heads: int, head_dim: int, cache_k=None, cache_v=None, n_threads: int = 1):
    """src/model.rs:232-254 middle section. Returns (out[t, hidden], new_cache_k, new_cache_v,
    q_roped, k_roped)."""
    hidden, kv_dim = n_heads * head_dim, n_kv_heads * head_dim
    q = _f32(q).reshape(-1).copy()
    k = _f32(k).reshape(-1).copy()
    v = _f32(v).reshape(-1)
    t = q.size // hidden
    base = 0 if cache_k is None else np.asarray(cache_k).size // kv_dim
    ck = np.zeros((base + t) * kv_dim + 1, np.float32)
    cv = np.zeros((base + t) * kv_dim + 1, np.float32)
    if base:
        ck[: base * kv_dim] = np.asarray(cache_k, np.float32).reshape(-1)
        cv[: base * kv_dim] = np.asarray(cache_v, np.float32).reshape(-1)
    n = C.c_size_t(base)
    out = np.zeros(t * hidden, np.float32)
    rc = lib().orc_attn_batch(q, k, v, t, pos0, _f32(q_gain), _f32(k_gain), theta, eps, n_heads,
                              n_kv_heads, head_dim, ck, cv, C.byref(n), out, n_threads)
    if rc:
        raise ValueError(f"oracle attn_batch failed: {rc}")
    m = n.value * kv_dim
    return (out.reshape(t, hidden), ck[:m].reshape(-1, kv_dim), cv[:m].reshape(-1, kv_dim),
            q.reshape(t, hidden), k.reshape(t, kv_dim))


# ------------------------------------------------------------------ cache --
class Cache:
    """Restatement of the attention part of ``src/cache.rs:9-49``: per layer a
    growable K and V history (``KV_DIM`` floats per position), ``pos`` (the next
    token's absolute position, never rewound by eviction)."""

    def __init__(self, n_layers: int, kv_dim: int = 512):
        self.kv_dim = kv_dim
        self.k = [np.zeros((0, kv_dim), np.float32) for _ in range(n_layers)]
        self.v = [np.zeros((0, kv_dim), np.float32) for _ in range(n_layers)]
        self.pos = 0

    def kv_len(self) -> int:  # src/cache.rs:33-35
        return max((k.shape[0] for k in self.k), default=0)

    def evict_front(self, n: int) -> None:  # src/cache.rs:40-48
        for l in range(len(self.k)):
            if self.k[l].shape[0] >= n:
                self.k[l] = self.k[l][n:]
                self.v[l] = self.v[l][n:]

    def append(self, layer: int, k, v) -> None:  # extend_from_slice, src/model.rs:443-444
        self.k[layer] = np.concatenate([self.k[layer], _f32(k).reshape(-1, self.kv_dim)])
        self.v[layer] = np.concatenate([self.v[layer], _f32(v).reshape(-1, self.kv_dim)])

    def clone(self) -> "Cache":  # #[derive(Clone)], src/cache.rs:9
        return copy.deepcopy(self)

    def attn_step(self, layer, q, k, v, q_gain, k_gain, theta, eps, n_heads, n_kv_heads, head_dim,
                  pos=None, n_threads=1):
        """src/model.rs:440-451 middle section on this cache; returns out[hidden]."""
        pos = self.pos if pos is None else pos
        q = norm_rope_heads(q, n_heads, head_dim, q_gain, pos, theta, eps)
        k = norm_rope_heads(k, n_kv_heads, head_dim, k_gain, pos, theta, eps)
        self.append(layer, k, v)
        n_ctx = self.k[layer].shape[0]
        return attention_decode(q, self.k[layer], self.v[layer], n_ctx, n_heads, n_kv_heads,
                                head_dim, n_threads=n_threads)


# ------------------------------------------------------------- quantized path --
# ggml type ids (src/tensor.rs:41-62)
GG_F32, GG_F16, GG_Q4_K, GG_Q6_K = 0, 1, 12, 14
BLOCK = {GG_F32: (1, 4), GG_F16: (1, 2), GG_Q4_K: (256, 144), GG_Q6_K: (256, 210)}


def f16_to_f32(h: int) -> float:
    """src/kernels/dequant.rs:22-54."""
    return float(lib().orc_f16_to_f32(int(h) & 0xFFFF))


def dequantize(dtype: int, data, n: int) -> np.ndarray:
    """src/kernels/dequant.rs:151-186: n elements of dtype from the raw bytes."""
    d = np.ascontiguousarray(np.frombuffer(bytes(data), np.uint8) if not isinstance(data, np.ndarray) else data,
                             np.uint8).reshape(-1)
    out = np.zeros(n, np.float32)
    if lib().orc_dequantize(dtype, d, n, out):
        raise ValueError(f"dequantize: unsupported dtype {dtype} or size {n}")
    return out


def quantize_q8(x):
    """src/kernels/matmul.rs:141-164 -> (q int8 [n], scales f32 [n/256], sums int32 [n/32])."""
    x = _f32(x).reshape(-1)
    q = np.zeros(x.size, np.int8)
    sc = np.zeros(x.size // 256, np.float32)
    sm = np.zeros(x.size // 32, np.int32)
    lib().orc_quantize_q8(x, x.size, q, sc, sm)
    return q, sc, sm


def matmul(dtype: int, w, n_in: int, n_out: int, x, n_tokens: int = 1) -> np.ndarray:
    """src/kernels/matmul.rs:850-1013: y [n_tokens][n_out] = W x, W packed as dtype (row per output)."""
    wb = np.ascontiguousarray(np.frombuffer(bytes(w), np.uint8) if not isinstance(w, np.ndarray) else w,
                              np.uint8).reshape(-1)
    x = _f32(x).reshape(-1)
    y = np.zeros(n_tokens * n_out, np.float32)
    scratch = np.zeros(max(n_in, 1), np.float32)
    q8 = np.zeros(max(n_in, 1), np.int8)
    q8s = np.zeros(max(n_in // 256, 1), np.float32)
    q8m = np.zeros(max(n_in // 32, 1), np.int32)
    if lib().orc_matmul(dtype, wb, n_in, n_out, x, n_tokens, y, scratch, q8, q8s, q8m):
        raise ValueError(f"matmul: unsupported dtype {dtype} or n_in {n_in}")
    return y.reshape(n_tokens, n_out) if n_tokens > 1 else y


def matvec(dtype: int, w, n_in: int, n_out: int, x) -> np.ndarray:
    return matmul(dtype, w, n_in, n_out, x, 1)


# ------------------------------------------------------- greedy token choice --
def argmax(x) -> int:
    """src/sampler.rs:139-149."""
    x = _f32(x)
    return int(lib().orc_argmax(x, x.size))


def sample_greedy(logits: np.ndarray, history=(), repeat_penalty: float = 1.0) -> int:
    """Sampler::sample with temperature <= 0 (src/sampler.rs:64-88); logits (float32) are
    rewritten in place by the penalty, as in the reference."""
    if logits.dtype != np.float32 or not logits.flags.c_contiguous:
        raise ValueError("logits must be a contiguous float32 array (rewritten in place)")
    h = np.ascontiguousarray(np.asarray(history, np.uint32).reshape(-1))
    tok = np.zeros(1, np.uint32)
    if lib().orc_sample_greedy(logits, logits.size, h, h.size, repeat_penalty, tok):
        raise ValueError("history token out of range")
    return int(tok[0])


def logits_head(dtype: int, token_embd, hidden: int, vocab: int, norm_gain, h, eps: float = 1e-5):
    """Model::logits_from_hidden (src/model.rs:379-388): rmsnorm, then the tied matvec."""
    return matvec(dtype, token_embd, hidden, vocab, rmsnorm(h, norm_gain, eps))
