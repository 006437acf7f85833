// Kernel 1: fused per-head RMSNorm + NEOX RoPE (+ paged KV append).
//
// Restates, per head of one position:
//   rmsnorm   src/kernels/rmsnorm.rs:10-21  (Σx² of f32 squares accumulated in f64,
//             mean narrowed to f32, scale = 1/sqrtf(mean+eps), out = (x*scale)*g)
//   rope_neox src/kernels/rope.rs:16-29     (split-half pairs, theta = pos, then
//             theta *= theta_scale after each pair; accurate sinf/cosf)
//   glue      src/model.rs:600-608 (norm_rope_heads) and the cache append of
//             src/model.rs:443-444 / 241-242.
// Every multiply/add that the reference performs unfused is written with the
// round-to-nearest intrinsics so the compiler cannot contract it into an FMA;
// with IEEE division and square root the only rounding differences left are
// those of sinf/cosf (a few ulp) and the f64 summation order (invisible after
// narrowing in practice).
//
// Mapping: 8 lanes per head (4 heads per warp). Lane `sub` owns pairs
// 4*sub .. 4*sub+3, i.e. elements x[4sub..4sub+3] and x[half+4sub..+3]; for
// head_dim 64 these are two float4 loads and two 128-bit stores per lane, so a
// head row moves as 256 contiguous bytes.
#include <algorithm>

#include "internal.h"

namespace bebelm {
namespace {

__device__ __forceinline__ void load_bf16x4(const __nv_bfloat16* p, float* out) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&u.x), b = *reinterpret_cast<const __nv_bfloat162*>(&u.y);
    out[0] = __low2float(a);
    out[1] = __high2float(a);
    out[2] = __low2float(b);
    out[3] = __high2float(b);
}

template <bool HD64>
__global__ void __launch_bounds__(256) norm_rope_kernel(NormRopeArgs a) {
    if (a.trigger_dependents) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int lane = threadIdx.x & 31;
    const int sub = lane & 7;
    const int nh_all = a.n_heads + a.n_kv;
    const long long total = (long long)a.T * nh_all;
    long long item = (long long)blockIdx.x * (blockDim.x >> 3) + (threadIdx.x >> 3);
    const bool active = item < total;
    if (!active) item = total - 1;  // keep the 8-lane group converged for the shuffles

    const int hd = HD64 ? 64 : a.head_dim;
    const int half = hd >> 1;
    // 32-bit division (a launch holds fewer than 2^31 head items; 64-bit division is emulated)
    const int tok = (int)((unsigned)item / (unsigned)nh_all);

    const int hh = (int)((unsigned)item - (unsigned)tok * (unsigned)nh_all);
    const bool is_q = hh < a.n_heads;
    const int head = is_q ? hh : hh - a.n_heads;
    const int q_row = a.q_row_heads ? a.q_row_heads : a.n_heads, kv_row = a.kv_row_heads ? a.kv_row_heads : a.n_kv;
    const size_t src_elem = is_q ? ((size_t)tok * q_row + a.q_head0 + head) * hd
                                 : ((size_t)tok * kv_row + a.kv_head0 + head) * hd;
    const float* src = a.in_bf16 ? reinterpret_cast<const float*>(
                                       reinterpret_cast<const __nv_bfloat16*>(is_q ? a.q : a.k) + src_elem)
                                 : (is_q ? a.q : a.k) + src_elem;
    const float* gain = is_q ? a.q_gain : a.k_gain;
    const bool do_norm = is_q ? (a.norm_q != 0) : (a.norm_k != 0);

    float x0[4], x1[4];
    if (HD64 && a.in_bf16) {
        const __nv_bfloat16* bsrc = reinterpret_cast<const __nv_bfloat16*>(src);
        load_bf16x4(bsrc + 4 * sub, x0);
        load_bf16x4(bsrc + 32 + 4 * sub, x1);
    } else if (HD64) {
        float4 u = *reinterpret_cast<const float4*>(src + 4 * sub);
        float4 w = *reinterpret_cast<const float4*>(src + 32 + 4 * sub);
        x0[0] = u.x; x0[1] = u.y; x0[2] = u.z; x0[3] = u.w;
        x1[0] = w.x; x1[1] = w.y; x1[2] = w.z; x1[3] = w.w;
    } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            int i = 4 * sub + e;
            x0[e] = i < half ? src[i] : 0.f;
            x1[e] = i < half ? src[i + half] : 0.f;
        }
    }

    // V row of the same kv head passes through unchanged (loaded now, stored at the end)
    const size_t v_elem = ((size_t)tok * kv_row + a.kv_head0 + head) * 64;
    const float* vsrc = !HD64 || is_q || !a.v ? nullptr
                        : a.in_bf16 ? reinterpret_cast<const float*>(reinterpret_cast<const __nv_bfloat16*>(a.v) + v_elem)
                                    : a.v + v_elem;
    float4 v0 = make_float4(0.f, 0.f, 0.f, 0.f), v1 = v0;
    if (vsrc && a.in_bf16) {
        const __nv_bfloat16* bv = reinterpret_cast<const __nv_bfloat16*>(vsrc);
        float t0[4], t1[4];
        load_bf16x4(bv + 4 * sub, t0);
        load_bf16x4(bv + 32 + 4 * sub, t1);
        v0 = make_float4(t0[0], t0[1], t0[2], t0[3]);
        v1 = make_float4(t1[0], t1[1], t1[2], t1[3]);
    } else if (vsrc) {
        v0 = *reinterpret_cast<const float4*>(vsrc + 4 * sub);
        v1 = *reinterpret_cast<const float4*>(vsrc + 32 + 4 * sub);
    }
    // RoPE angles depend only on (position, pair): every head of a token shares them, so the
    // block builds cos/sin once per token it touches (at most 32 tokens: 32 items per block),
    // with the reference's iterative angle, theta = pos * scale^i by repeated multiplication.
    // It does so after issuing its loads, so their latency overlaps the table.
    __shared__ float s_cos[32][32], s_sin[32][32];
    const long long item0 = (long long)blockIdx.x * (blockDim.x >> 3);
    const int tok0 = (int)((unsigned)item0 / (unsigned)nh_all);
    if (a.norm_q || a.norm_k) {
        const long long item_last = min(total - 1, item0 + (blockDim.x >> 3) - 1);
        const int ntok = (int)((unsigned)item_last / (unsigned)nh_all) - tok0 + 1;
        for (int idx = threadIdx.x; idx < ntok * half; idx += blockDim.x) {
            const int t = HD64 ? idx >> 5 : idx / half, i = HD64 ? idx & 31 : idx % half;
            const long long pos = a.targets ? a.targets[tok0 + t].pos : a.pos0 + tok0 + t;
            float theta = __ll2float_rn(pos);
            for (int r = 0; r < i; ++r) theta = __fmul_rn(theta, a.theta_scale);
            s_cos[t][i] = cosf(theta);
            s_sin[t][i] = sinf(theta);
        }
        __syncthreads();
    }
    if (do_norm) {
        double ss = 0.0;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            ss += (double)__fmul_rn(x0[e], x0[e]);
            ss += (double)__fmul_rn(x1[e], x1[e]);
        }
        ss += __shfl_xor_sync(0xffffffffu, ss, 1);
        ss += __shfl_xor_sync(0xffffffffu, ss, 2);
        ss += __shfl_xor_sync(0xffffffffu, ss, 4);
        const float mean = __double2float_rn(ss / (double)hd);
        const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, a.eps)));
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            int i = 4 * sub + e;
            if (HD64 || i < half) {
                x0[e] = __fmul_rn(__fmul_rn(x0[e], scale), gain[i]);
                x1[e] = __fmul_rn(__fmul_rn(x1[e], scale), gain[i + half]);
            }
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            int i = 4 * sub + e;
            if (HD64 || i < half) {
                const float sn = s_sin[tok - tok0][i], cs = s_cos[tok - tok0][i];
                const float p = x0[e], q = x1[e];
                x0[e] = __fsub_rn(__fmul_rn(p, cs), __fmul_rn(q, sn));
                x1[e] = __fadd_rn(__fmul_rn(p, sn), __fmul_rn(q, cs));
            }
        }
    }
    if (!active) return;

    float* dst = nullptr;
    if (is_q) {
        dst = a.q_out ? a.q_out + ((size_t)tok * a.n_heads + head) * hd : nullptr;
    } else {
        dst = a.k_out ? a.k_out + ((size_t)tok * a.n_kv + head) * hd : nullptr;
    }
    if (dst) {
        if (HD64) {
            *reinterpret_cast<float4*>(dst + 4 * sub) = make_float4(x0[0], x0[1], x0[2], x0[3]);
            *reinterpret_cast<float4*>(dst + 32 + 4 * sub) = make_float4(x1[0], x1[1], x1[2], x1[3]);
        } else {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                int i = 4 * sub + e;
                if (i < half) {
                    dst[i] = x0[e];
                    dst[i + half] = x1[e];
                }
            }
        }
    }
    if (!HD64) return;

    // bf16 copies for the tensor-core prefill
    __nv_bfloat16* bdst = is_q ? (a.q_bf16 ? a.q_bf16 + ((size_t)tok * a.n_heads + head) * 64 : nullptr)
                               : (a.k_bf16 ? a.k_bf16 + ((size_t)tok * a.n_kv + head) * 64 : nullptr);
    if (bdst) {
        __nv_bfloat162 b0 = __floats2bfloat162_rn(x0[0], x0[1]), b1 = __floats2bfloat162_rn(x0[2], x0[3]);
        __nv_bfloat162 b2 = __floats2bfloat162_rn(x1[0], x1[1]), b3 = __floats2bfloat162_rn(x1[2], x1[3]);
        uint2 lo, hi;
        lo.x = *reinterpret_cast<uint32_t*>(&b0); lo.y = *reinterpret_cast<uint32_t*>(&b1);
        hi.x = *reinterpret_cast<uint32_t*>(&b2); hi.y = *reinterpret_cast<uint32_t*>(&b3);
        *reinterpret_cast<uint2*>(bdst + 4 * sub) = lo;
        *reinterpret_cast<uint2*>(bdst + 32 + 4 * sub) = hi;
    }
    if (is_q) return;

    if (a.v_bf16 && vsrc) {
        __nv_bfloat16* vb = a.v_bf16 + ((size_t)tok * a.n_kv + head) * 64;
        __nv_bfloat162 b0 = __floats2bfloat162_rn(v0.x, v0.y), b1 = __floats2bfloat162_rn(v0.z, v0.w);
        __nv_bfloat162 b2 = __floats2bfloat162_rn(v1.x, v1.y), b3 = __floats2bfloat162_rn(v1.z, v1.w);
        uint2 lo, hi;
        lo.x = *reinterpret_cast<uint32_t*>(&b0); lo.y = *reinterpret_cast<uint32_t*>(&b1);
        hi.x = *reinterpret_cast<uint32_t*>(&b2); hi.y = *reinterpret_cast<uint32_t*>(&b3);
        *reinterpret_cast<uint2*>(vb + 4 * sub) = lo;
        *reinterpret_cast<uint2*>(vb + 32 + 4 * sub) = hi;
    }
    if (a.append) {
        const int* table = a.targets ? a.targets[tok].table : a.table;
        const int cap = a.targets ? a.targets[tok].cap : a.cap;
        const long long slot = a.targets ? a.targets[tok].slot : a.slot0 + tok;
        const size_t kd = slot_offset(a.pv, table, cap, slot, head, 0);
        const size_t vd = kd + a.pv.block_bytes;  // the V row of the same slot and head
        kv_store4(a.pv, kd, 4 * sub, make_float4(x0[0], x0[1], x0[2], x0[3]));
        kv_store4(a.pv, kd, 32 + 4 * sub, make_float4(x1[0], x1[1], x1[2], x1[3]));
        kv_store4(a.pv, vd, 4 * sub, v0);
        kv_store4(a.pv, vd, 32 + 4 * sub, v1);
    }
}

// One warp per (token, kv head) row: 16 lanes x float4 for K, then for V.
__global__ void __launch_bounds__(256) kv_gather_kernel(PoolView pv, const int* table, int cap, long long base,
                                                        long long len, int n_kv, float* k_out, float* v_out) {
    const long long row = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
    if (row >= len * n_kv) return;
    const int lane = threadIdx.x & 31;
    const long long t = row / n_kv;
    const int h = (int)(row % n_kv);
    const int kind = lane >> 4;  // lanes 0-15: K, 16-31: V
    float* dst = kind ? v_out : k_out;
    if (!dst) return;
    const size_t src = slot_offset(pv, table, cap, base + t, h, kind);
    const int e = (lane & 15) * 4;
    *reinterpret_cast<float4*>(dst + (size_t)row * 64 + e) = kv_load4(pv, src, e);
}

// One thread per 4 consecutive floats of the [len][n_kv][64] window, K and V.
__global__ void kv_gather_bf16_kernel(PoolView pv, const int* table, int cap, long long base, long long len, int n_kv,
                                      __nv_bfloat16* k_out, __nv_bfloat16* v_out) {
    const long long quads = len * n_kv * 16;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < quads;
         i += (long long)gridDim.x * blockDim.x) {
        const long long row = i >> 4;
        const int e = (int)(i & 15) * 4;
        const long long t = row / n_kv;
        const int h = (int)(row % n_kv);
        const size_t ko = slot_offset(pv, table, cap, base + t, h, 0);
        const float4 kf = kv_load4(pv, ko, e);
        const float4 vf = kv_load4(pv, ko + pv.block_bytes, e);
        __nv_bfloat162 k0 = __floats2bfloat162_rn(kf.x, kf.y), k1 = __floats2bfloat162_rn(kf.z, kf.w);
        __nv_bfloat162 v0 = __floats2bfloat162_rn(vf.x, vf.y), v1 = __floats2bfloat162_rn(vf.z, vf.w);
        uint2 kw, vw;
        kw.x = *reinterpret_cast<uint32_t*>(&k0); kw.y = *reinterpret_cast<uint32_t*>(&k1);
        vw.x = *reinterpret_cast<uint32_t*>(&v0); vw.y = *reinterpret_cast<uint32_t*>(&v1);
        *reinterpret_cast<uint2*>(k_out + row * 64 + e) = kw;
        *reinterpret_cast<uint2*>(v_out + row * 64 + e) = vw;
    }
}


}  // namespace

cudaError_t launch_kv_gather(const PoolView& pv, const int* table, int cap, long long base, long long len,
                             int n_kv, float* k_out, float* v_out, cudaStream_t s) {
    const long long rows = len * n_kv;
    if (rows <= 0) return cudaSuccess;
    kv_gather_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, s>>>(pv, table, cap, base, len, n_kv, k_out, v_out);
    return cudaGetLastError();
}

cudaError_t launch_kv_gather_bf16(const PoolView& pv, const int* table, int cap, long long base, long long len,
                                  int n_kv, __nv_bfloat16* k_out, __nv_bfloat16* v_out, cudaStream_t s) {
    const long long quads = len * n_kv * 16;
    if (quads <= 0) return cudaSuccess;
    const long long blocks = std::min<long long>((quads + 255) / 256, 148 * 16);
    kv_gather_bf16_kernel<<<(unsigned)blocks, 256, 0, s>>>(pv, table, cap, base, len, n_kv, k_out, v_out);
    return cudaGetLastError();
}

cudaError_t launch_norm_rope(const NormRopeArgs& a, cudaStream_t s) {
    const long long items = (long long)a.T * (a.n_heads + a.n_kv);
    if (items <= 0) return cudaSuccess;
    if (items >= (1ll << 31)) return cudaErrorInvalidValue;  // the kernel indexes items in 32 bits
    const int heads_per_block = 256 / 8;
    const long long blocks = (items + heads_per_block - 1) / heads_per_block;
    if (a.head_dim == 64)
        norm_rope_kernel<true><<<(unsigned)blocks, 256, 0, s>>>(a);
    else
        norm_rope_kernel<false><<<(unsigned)blocks, 256, 0, s>>>(a);
    return cudaGetLastError();
}

}  // namespace bebelm
