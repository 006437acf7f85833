// Quantized weights feeding the attention path: GGML dequantization and the quantized
// matrix-vector / matrix-matrix product of the reference (its q/k/v/o projections).
//
// Restates, per output row and token, the reference's arithmetic exactly:
//   quantize_q8       src/kernels/matmul.rs:141-164  activations -> int8 per 256-block:
//                     scale = max|x|/127, q = round_half_away(x * 127/max|x|) clamped to +-127,
//                     plus the sum of each 32-wide sub-block's quants
//   dot_q4k_block_q8  src/kernels/matmul.rs:220-244  exact i32 Σ_j sc_j·<nibbles_j, q_j> and
//                     Σ_j m_j·sum_j, then sx * (d * sd - dmin * sm) in f32 (no contraction)
//   dot_q6k_block_q8  src/kernels/matmul.rs:633-700  exact i32 Σ_k sc_k·<(q6 - 32)_k, q_k>, then
//                     sx * (d * s)
//   dot_q{4,6}k_row   src/kernels/matmul.rs:293-300, 748-754  f32 sum over blocks in order
//   matvec / matmul   src/kernels/matmul.rs:850-1013  (matmul = matvec per token, bit for bit)
//   F32/F16 weights:  the row dequantized, then `dot` (src/kernels/matmul.rs:36-65): 32 FMA
//                     chains (lane = i mod 32), the 8-wide cleanup into the first 8, then
//                     ((acc0+acc1)+(acc2+acc3)) and an 8-lane reduction, then an unfused
//                     scalar tail. The 8-lane reduction order of the reference's SIMD library
//                     is not visible; the order here is the CPU oracle's.
//   dequantize_*      src/kernels/dequant.rs:22-176
// The integer dots are exact and every f32 operation is written with round-to-nearest
// intrinsics in the reference's order, so Q4_K/Q6_K results are the reference's bit for bit.
//
// Mapping: one warp per (output row, token); a 256-weight block per step, 8 weights per lane
// (dp4a on packed int8), an exact integer warp reduction, and lane 0 adds the block's f32
// value to the row's sum in block order. Activations are quantized once per token by a
// separate kernel (one warp per 256-block).
#include <algorithm>

#include <math_constants.h>

#include <cstdlib>

#include "internal.h"

namespace bebelm {
namespace {

constexpr int kQK = 256;
#ifndef BEBELM_QMM_TILED_MIN
#define BEBELM_QMM_TILED_MIN 32
#endif
constexpr size_t kTiledMinTokens = BEBELM_QMM_TILED_MIN;  // from this many tokens on, the tiled kernel
constexpr size_t kTcMinTokens = 64;  // from this many tokens on, K-quants go to the tensor cores

__device__ __forceinline__ float f16_bits_to_f32(uint32_t h) {
    // exact for normals, subnormals, inf and nan (the hardware conversion is exact)
    __half_raw r;
    r.x = (unsigned short)h;
    return __half2float(__half(r));
}

__device__ __forceinline__ float ld_f16(const uint8_t* p) {
    return f16_bits_to_f32((uint32_t)p[0] | ((uint32_t)p[1] << 8));
}

__device__ __forceinline__ void scale_min_k4(int j, const uint8_t* s, int& sc, int& m) {
    if (j < 4) {
        sc = s[j] & 63;
        m = s[j + 4] & 63;
    } else {
        sc = (s[j + 4] & 0x0f) | ((s[j - 4] >> 6) << 4);
        m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

__device__ __forceinline__ int warp_sum_i32(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// One warp per 256-block of one token.
__global__ void __launch_bounds__(256) quantize_q8_kernel(const float* x, size_t n_in, int8_t* q, float* scales,
                                                          int* sums, size_t n_blocks_total) {
    const size_t blk = (size_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    if (blk >= n_blocks_total) return;
    const int lane = threadIdx.x & 31;
    const float* xb = x + blk * kQK + lane * 8;
    const float4 a = *reinterpret_cast<const float4*>(xb), b = *reinterpret_cast<const float4*>(xb + 4);
    const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float inv = amax > 0.f ? __fdiv_rn(127.0f, amax) : 0.f;
    int8_t qv[8];
    int s = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        float r = roundf(__fmul_rn(v[i], inv));  // half away from zero, as Rust's f32::round
        r = fminf(fmaxf(r, -127.f), 127.f);
        qv[i] = (int8_t)r;
        s += qv[i];
    }
    *reinterpret_cast<uint2*>(q + blk * kQK + lane * 8) = *reinterpret_cast<const uint2*>(qv);
    s += __shfl_xor_sync(0xffffffffu, s, 1);  // a 32-wide sub-block is 4 lanes
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    if ((lane & 3) == 0) sums[blk * 8 + (lane >> 2)] = s;
    if (lane == 0) scales[blk] = __fdiv_rn(amax, 127.0f);
}

// One 256-weight block for one warp, split into the loads and the arithmetic so the one-token
// kernel can issue several blocks' loads before using any.
// Q4_K block (144 B: d, dmin, scales[12], qs[128]): lane l holds qs bytes 4l..4l+3, chunk
// c = l/8 (sub-blocks 2c: low nibbles, 2c+1: high).
struct Q4Ld {
    uint4 head;  // d, dmin, scales[12]
    uint32_t w;
    int xlo, xhi, sum;
    float sx;
};
__device__ __forceinline__ Q4Ld load_q4k(const uint8_t* blk, const int8_t* qx, float sx, const int* sums, int lane) {
    const int c = lane >> 3, p = (lane & 7) * 4;
    Q4Ld L;
    L.head = *reinterpret_cast<const uint4*>(blk);
    L.w = *reinterpret_cast<const uint32_t*>(blk + 16 + c * 32 + p);
    L.xlo = *reinterpret_cast<const int*>(qx + (2 * c) * 32 + p);
    L.xhi = *reinterpret_cast<const int*>(qx + (2 * c + 1) * 32 + p);
    L.sum = lane < 8 ? sums[lane] : 0;
    L.sx = sx;
    return L;
}
// byte j of the 16-byte block head
__device__ __forceinline__ int head_byte(const uint4& h, int j) {
    const uint32_t w = j < 4 ? h.x : j < 8 ? h.y : j < 12 ? h.z : h.w;
    return (int)((w >> (8 * (j & 3))) & 0xffu);
}
// get_scale_min_k4 on the scales held in the head's bytes 4..15
__device__ __forceinline__ void scale_min_head(int j, const uint4& h, int& sc, int& m) {
    if (j < 4) {
        sc = head_byte(h, 4 + j) & 63;
        m = head_byte(h, 8 + j) & 63;
    } else {
        sc = (head_byte(h, 8 + j) & 0x0f) | ((head_byte(h, j) >> 6) << 4);
        m = (head_byte(h, 8 + j) >> 4) | ((head_byte(h, 4 + j) >> 6) << 4);
    }
}
__device__ __forceinline__ float dot_q4k(const Q4Ld& L, int lane) {
    const int c = lane >> 3;
    int sc0, m0, sc1, m1;
    scale_min_head(2 * c, L.head, sc0, m0);
    scale_min_head(2 * c + 1, L.head, sc1, m1);
    int sd = sc0 * __dp4a((int)(L.w & 0x0f0f0f0fu), L.xlo, 0) + sc1 * __dp4a((int)((L.w >> 4) & 0x0f0f0f0fu), L.xhi, 0);
    int sm = 0;
    if (lane < 8) {
        int scj, mj;
        scale_min_head(lane, L.head, scj, mj);
        sm = mj * L.sum;
    }
    sd = warp_sum_i32(sd);
    sm = warp_sum_i32(sm);
    const float d = f16_bits_to_f32(L.head.x & 0xffffu), dmin = f16_bits_to_f32(L.head.x >> 16);
    return __fmul_rn(L.sx, __fsub_rn(__fmul_rn(d, __int2float_rn(sd)), __fmul_rn(dmin, __int2float_rn(sm))));
}

// Q6_K block (210 B: ql[128], qh[64], scales[16] i8, d): lane l holds 8 weights of the
// 16-wide sub-block k = l/2, the low 4 bits from ql (low or high nibble), the top 2 from qh.
struct Q6Ld {
    uint32_t ql[2], qh[2];  // 8 bytes each, little-endian
    int x0, x1, sc;
    uint32_t dbits;
    float sx;
};
__device__ __forceinline__ Q6Ld load_q6k(const uint8_t* blk, const int8_t* qx, float sx, int lane) {
    const int k = lane >> 1, h = lane & 1;
    const int n = k >> 3, g = (k & 7) >> 1, sub = k & 1;
    const int ql_off = n * 64 + (g & 1) * 32 + sub * 16 + h * 8, qh_off = 128 + n * 32 + sub * 16 + h * 8;
    Q6Ld L;
#pragma unroll
    for (int part = 0; part < 2; ++part) {
        uint32_t a = 0, b = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            a |= (uint32_t)blk[ql_off + 4 * part + i] << (8 * i);
            b |= (uint32_t)blk[qh_off + 4 * part + i] << (8 * i);
        }
        L.ql[part] = a;
        L.qh[part] = b;
    }
    const int8_t* x = qx + k * 16 + h * 8;
    L.x0 = *reinterpret_cast<const int*>(x);
    L.x1 = *reinterpret_cast<const int*>(x + 4);
    L.sc = (int)(int8_t)blk[192 + k];
    L.dbits = (uint32_t)blk[208] | ((uint32_t)blk[209] << 8);
    L.sx = sx;
    return L;
}
__device__ __forceinline__ float dot_q6k(const Q6Ld& L, int lane) {
    const int k = lane >> 1, g = (k & 7) >> 1;
    const bool high = g >= 2;
    const int shift = 2 * g;
    uint32_t wq[2];
#pragma unroll
    for (int part = 0; part < 2; ++part) {
        uint32_t word = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t l = (L.ql[part] >> (8 * i)) & 0xffu, hb = ((L.qh[part] >> (8 * i)) >> shift) & 3u;
            word |= ((((high ? (l >> 4) : (l & 0x0fu)) | (hb << 4)) - 32u) & 0xffu) << (8 * i);
        }
        wq[part] = word;
    }
    int t = __dp4a((int)wq[0], L.x0, 0);
    t = __dp4a((int)wq[1], L.x1, t);
    const int s = warp_sum_i32(t * L.sc);
    return __fmul_rn(L.sx, __fmul_rn(f16_bits_to_f32(L.dbits), __int2float_rn(s)));
}

// F32/F16 weight row against fp32 x: the reference's `dot` (see the file header).
template <int DT>
__device__ __forceinline__ float row_dot(const uint8_t* row, const float* x, size_t n, int lane) {
    auto wv = [&](size_t i) -> float {
        return DT == kGgmlF32 ? reinterpret_cast<const float*>(row)[i] : ld_f16(row + 2 * i);
    };
    float acc = 0.f;
    size_t i = 0;
    for (; i + 32 <= n; i += 32) acc = fmaf(wv(i + lane), x[i + lane], acc);
    for (; i + 8 <= n; i += 8)
        if (lane < 8) acc = fmaf(wv(i + lane), x[i + lane], acc);
    acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 8));   // acc0+acc1, acc2+acc3
    acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 16));  // (acc0+acc1)+(acc2+acc3)
    acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 4));   // lanes j and j+4
    acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 2));   // (0,2), (1,3)
    acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 1));   // the two halves
    if (lane == 0)
        for (; i < n; ++i) acc = __fadd_rn(acc, __fmul_rn(wv(i), x[i]));
    return acc;
}

// grid (ceil(n_out/8), n_tokens), 8 warps: warp = one output row of one token.
template <int DT>
__global__ void __launch_bounds__(256) qmatmul_kernel(const uint8_t* w, size_t row_bytes, size_t n_in, size_t n_out,
                                                      const float* x, const int8_t* q8, const float* q8_scales,
                                                      const int* q8_sums, float* y) {
    const size_t o = (size_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    if (o >= n_out) return;
    const int lane = threadIdx.x & 31;
    const size_t t = blockIdx.y;
    const uint8_t* row = w + o * row_bytes;
    float acc;
    if (DT == kGgmlQ4K || DT == kGgmlQ6K) {
        const size_t nb = n_in / kQK;
        const int8_t* qx = q8 + t * n_in;
        const float* sx = q8_scales + t * nb;
        acc = -0.0f;  // an f32 iterator sum over the blocks, in order
        // up to 8 blocks' loads are issued before any of them is used, so a row costs one
        // memory round trip per 8 blocks instead of one per block
        constexpr int kU = 8;
        for (size_t b0 = 0; b0 < nb; b0 += kU) {
            if (DT == kGgmlQ4K) {
                Q4Ld L[kU];
#pragma unroll
                for (int u = 0; u < kU; ++u)
                    if (b0 + u < nb)
                        L[u] = load_q4k(row + (b0 + u) * 144, qx + (b0 + u) * kQK, sx[b0 + u],
                                        q8_sums + (t * nb + b0 + u) * 8, lane);
#pragma unroll
                for (int u = 0; u < kU; ++u)
                    if (b0 + u < nb) acc = __fadd_rn(acc, dot_q4k(L[u], lane));
            } else {
                Q6Ld L[kU];
#pragma unroll
                for (int u = 0; u < kU; ++u)
                    if (b0 + u < nb) L[u] = load_q6k(row + (b0 + u) * 210, qx + (b0 + u) * kQK, sx[b0 + u], lane);
#pragma unroll
                for (int u = 0; u < kU; ++u)
                    if (b0 + u < nb) acc = __fadd_rn(acc, dot_q6k(L[u], lane));
            }
        }
    } else {
        acc = row_dot<DT>(row, x + t * n_in, n_in, lane);
    }
    if (lane == 0) y[t * n_out + o] = acc;
}

// Many tokens: a CTA computes 64 rows x 64 tokens. For each 256-weight block it unpacks the
// 64 rows' weights to int8 in shared memory (Q4_K: nibbles 0..15 in 8 sub-blocks of 32;
// Q6_K: q - 32 in 16 sub-blocks of 16) with their integer sub-block scales, stages the 64
// tokens' Q8 activations, and each thread forms 4 rows x 4 tokens of exact integer sub-block
// dots with dp4a. The f32 block value and the in-order block sum per (row, token) are those
// of qmatmul_kernel, so the results are identical.
constexpr int kTR = 64, kTT = 64, kWStride = 256 + 16;  // int8 row stride: 16 B skew against bank conflicts
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
    const uint32_t sa = (uint32_t)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(sa), "l"(gmem), "r"(valid ? 16 : 0) : "memory");
}
__device__ __forceinline__ void cp_async4(void* smem, const void* gmem, bool valid) {
    const uint32_t sa = (uint32_t)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(sa), "l"(gmem), "r"(valid ? 4 : 0) : "memory");
}

// dynamic shared memory of the tiled kernel: two stages of the tokens' Q8 activations and (Q4_K)
// of the rows' raw block bytes, filled with cp.async while the other stage is computed on
constexpr int kTiledDynBytes = 2 * kTT * kWStride + 2 * kTR * 144;

template <int DT>
__global__ void __launch_bounds__(256) qmatmul_tiled_kernel(const uint8_t* w, size_t row_bytes, size_t n_in,
                                                            size_t n_out, size_t n_tokens, const int8_t* q8,
                                                            const float* q8_scales, const int* q8_sums, float* y) {
    constexpr int NSUB = DT == kGgmlQ4K ? 8 : 16;  // sub-blocks per block
    constexpr int SW = kQK / NSUB;                 // sub-block width (32 or 16)
    extern __shared__ __align__(16) uint8_t s_dyn[];
    int8_t* const s_x2 = reinterpret_cast<int8_t*>(s_dyn);          // [2][kTT][kWStride]
    uint8_t* const s_wraw = s_dyn + 2 * kTT * kWStride;             // [2][kTR][144] (Q4_K)
    __shared__ __align__(16) int8_t s_w[kTR * kWStride];
    __shared__ int s_sc[kTR][NSUB];
    __shared__ int s_m[kTR][8];       // Q4_K mins
    __shared__ float s_d[kTR], s_dmin[kTR];
    __shared__ __align__(16) float s_sx2[2][kTT];
    __shared__ __align__(16) int s_sums2[2][kTT][8];
    const int tid = threadIdx.x;
    const size_t r0 = (size_t)blockIdx.x * kTR, t0 = (size_t)blockIdx.y * kTT;
    const int tr = tid >> 4, tc = tid & 15;  // thread tile: rows tr + 16 i, tokens tc + 16 k
    const size_t nb = n_in / kQK;
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int k = 0; k < 4; ++k) acc[i][k] = -0.0f;

    // block bb's activations (and Q4_K raw weights) into stage st, asynchronously
    auto stage = [&](size_t bb, int st) {
        int8_t* sx = s_x2 + st * kTT * kWStride;
        for (int task = tid; task < kTT * 16; task += 256) {
            const int t = task >> 4, seg = task & 15;
            const bool ok = t0 + t < n_tokens;
            cp_async16(sx + t * kWStride + seg * 16, ok ? q8 + (t0 + t) * n_in + bb * kQK + seg * 16 : q8, ok);
        }
        if (tid < kTT) {
            const bool ok = t0 + tid < n_tokens;
            cp_async4(&s_sx2[st][tid], ok ? q8_scales + (t0 + tid) * nb + bb : q8_scales, ok);
            if (DT == kGgmlQ4K) {
                const int* src = ok ? q8_sums + ((t0 + tid) * nb + bb) * 8 : q8_sums;
                cp_async16(&s_sums2[st][tid][0], src, ok);
                cp_async16(&s_sums2[st][tid][4], ok ? src + 4 : q8_sums, ok);
            }
        }
        if (DT == kGgmlQ4K) {
            uint8_t* wr = s_wraw + st * kTR * 144;
            for (int task = tid; task < kTR * 9; task += 256) {
                const int r = task / 9, seg = task % 9;
                const bool ok = r0 + r < n_out;
                cp_async16(wr + r * 144 + seg * 16, ok ? w + (r0 + r) * row_bytes + bb * 144 + seg * 16 : w, ok);
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };

    stage(0, 0);
    for (size_t b = 0; b < nb; ++b) {
        const int st = (int)(b & 1);
        __syncthreads();  // the previous block's operands are no longer read
        if (b + 1 < nb)
            stage(b + 1, st ^ 1);
        else
            asm volatile("cp.async.commit_group;" ::: "memory");  // keep one group per iteration
        asm volatile("cp.async.wait_group 1;" ::: "memory");     // block b's copies have landed
        __syncthreads();
        const int8_t* s_x = s_x2 + st * kTT * kWStride;
        const float* s_sx = s_sx2[st];
        int (*s_sums)[8] = s_sums2[st];
        // weights of 64 rows -> int8 + scales
        if (DT == kGgmlQ4K) {
            for (int task = tid; task < kTR * 8; task += 256) {  // (row, 16-byte segment of qs)
                const int r = task >> 3, seg = task & 7, c = seg >> 1, p = (seg & 1) * 16;
                const uint4 q = *reinterpret_cast<const uint4*>(s_wraw + st * kTR * 144 + r * 144 + 16 + c * 32 + p);
                const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
                uint4 lo, hi;
                uint32_t* lp = reinterpret_cast<uint32_t*>(&lo);
                uint32_t* hp = reinterpret_cast<uint32_t*>(&hi);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    lp[e] = qw[e] & 0x0f0f0f0fu;
                    hp[e] = (qw[e] >> 4) & 0x0f0f0f0fu;
                }
                *reinterpret_cast<uint4*>(s_w + r * kWStride + (2 * c) * 32 + p) = lo;
                *reinterpret_cast<uint4*>(s_w + r * kWStride + (2 * c + 1) * 32 + p) = hi;
            }
            if (tid < kTR) {
                const int r = tid;
                if (r0 + r < n_out) {
                    const uint8_t* blk = s_wraw + st * kTR * 144 + r * 144;
#pragma unroll
                    for (int j = 0; j < 8; ++j) scale_min_k4(j, blk + 4, s_sc[r][j], s_m[r][j]);
                    s_d[r] = ld_f16(blk);
                    s_dmin[r] = ld_f16(blk + 2);
                } else {
#pragma unroll
                    for (int j = 0; j < 8; ++j) s_sc[r][j] = s_m[r][j] = 0;
                    s_d[r] = s_dmin[r] = 0.f;
                }
            }
        } else {  // Q6_K: (row, sub-block k, half h): 8 weights
            for (int task = tid; task < kTR * 32; task += 256) {
                const int r = task >> 5, k = (task >> 1) & 15, h = task & 1;
                uint2 out = make_uint2(0, 0);
                if (r0 + r < n_out) {
                    const uint8_t* blk = w + (r0 + r) * row_bytes + b * 210;
                    const int n = k >> 3, g = (k & 7) >> 1, sub = k & 1;
                    const int ql_off = n * 64 + (g & 1) * 32 + sub * 16 + h * 8;
                    const int qh_off = 128 + n * 32 + sub * 16 + h * 8;
                    const bool high = g >= 2;
                    const int shift = 2 * g;
                    uint32_t* op = reinterpret_cast<uint32_t*>(&out);
#pragma unroll
                    for (int part = 0; part < 2; ++part) {
                        uint32_t word = 0;
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const uint32_t l = blk[ql_off + part * 4 + i];
                            const uint32_t hb = (blk[qh_off + part * 4 + i] >> shift) & 3u;
                            word |= ((((high ? (l >> 4) : (l & 0x0fu)) | (hb << 4)) - 32u) & 0xffu) << (8 * i);
                        }
                        op[part] = word;
                    }
                }
                *reinterpret_cast<uint2*>(s_w + r * kWStride + k * 16 + h * 8) = out;
            }
            if (tid < kTR) {
                const int r = tid;
                const bool ok = r0 + r < n_out;
                const uint8_t* blk = w + (ok ? (r0 + r) * row_bytes + b * 210 : 0);
#pragma unroll
                for (int k = 0; k < 16; ++k) s_sc[r][k] = ok ? (int)(int8_t)blk[192 + k] : 0;
                s_d[r] = ok ? ld_f16(blk + 208) : 0.f;
            }
        }
        __syncthreads();

        int sd[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int k = 0; k < 4; ++k) sd[i][k] = 0;
#pragma unroll 2
        for (int j = 0; j < NSUB; ++j) {
            int wv[4][SW / 4], xv[4][SW / 4];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int q = 0; q < SW / 16; ++q)
                    *reinterpret_cast<int4*>(&wv[i][4 * q]) =
                        *reinterpret_cast<const int4*>(s_w + (tr + 16 * i) * kWStride + j * SW + 16 * q);
#pragma unroll
            for (int k = 0; k < 4; ++k)
#pragma unroll
                for (int q = 0; q < SW / 16; ++q)
                    *reinterpret_cast<int4*>(&xv[k][4 * q]) =
                        *reinterpret_cast<const int4*>(s_x + (tc + 16 * k) * kWStride + j * SW + 16 * q);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int sc = s_sc[tr + 16 * i][j];
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    int dt = 0;
#pragma unroll
                    for (int e = 0; e < SW / 4; ++e) dt = __dp4a(wv[i][e], xv[k][e], dt);
                    sd[i][k] += sc * dt;
                }
            }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int r = tr + 16 * i;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int t = tc + 16 * k;
                float v;
                if (DT == kGgmlQ4K) {
                    int sm = 0;
#pragma unroll
                    for (int j = 0; j < 8; ++j) sm += s_m[r][j] * s_sums[t][j];
                    v = __fmul_rn(s_sx[t], __fsub_rn(__fmul_rn(s_d[r], __int2float_rn(sd[i][k])),
                                                     __fmul_rn(s_dmin[r], __int2float_rn(sm))));
                } else {
                    v = __fmul_rn(s_sx[t], __fmul_rn(s_d[r], __int2float_rn(sd[i][k])));
                }
                acc[i][k] = __fadd_rn(acc[i][k], v);
            }
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const size_t r = r0 + tr + 16 * i, t = t0 + tc + 16 * k;
            if (r < n_out && t < n_tokens) y[t * n_out + r] = acc[i][k];
        }
}

// One token through up to three matrices of the same input in one launch (the q/k/v
// projections, or W_o alone): every CTA first quantizes x to Q8 in shared memory (the
// arithmetic of quantize_q8_kernel, so the quants are the same), then each warp computes one
// output row of one segment as qmatmul_kernel does. Saves the separate quantization launch and
// one launch per extra matrix.
constexpr int kMvMaxIn = 8192;  // x held in shared memory as int8
__global__ void __launch_bounds__(256) qmv_multi_kernel(QmvSegs segs, const float* x, size_t n_in) {
    __shared__ __align__(16) int8_t s_q[kMvMaxIn];
    __shared__ float s_sc[kMvMaxIn / kQK];
    __shared__ int s_sum[kMvMaxIn / 32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const size_t nb = n_in / kQK;
    bool kq = false;
    for (int i = 0; i < segs.n; ++i) kq |= segs.dtype[i] == kGgmlQ4K || segs.dtype[i] == kGgmlQ6K;
    if (kq) {
        for (size_t blk = warp; blk < nb; blk += 8) {
            const float* xb = x + blk * kQK + lane * 8;
            const float4 a = *reinterpret_cast<const float4*>(xb), b = *reinterpret_cast<const float4*>(xb + 4);
            const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
            float amax = 0.f;
#pragma unroll
            for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
            const float inv = amax > 0.f ? __fdiv_rn(127.0f, amax) : 0.f;
            int8_t qv[8];
            int sm = 0;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                float r = roundf(__fmul_rn(v[i], inv));
                r = fminf(fmaxf(r, -127.f), 127.f);
                qv[i] = (int8_t)r;
                sm += qv[i];
            }
            *reinterpret_cast<uint2*>(s_q + blk * kQK + lane * 8) = *reinterpret_cast<const uint2*>(qv);
            sm += __shfl_xor_sync(0xffffffffu, sm, 1);
            sm += __shfl_xor_sync(0xffffffffu, sm, 2);
            if ((lane & 3) == 0) s_sum[blk * 8 + (lane >> 2)] = sm;
            if (lane == 0) s_sc[blk] = __fdiv_rn(amax, 127.0f);
        }
        __syncthreads();
    }
    // which segment and row this warp computes
    size_t r = (size_t)blockIdx.x * 8 + warp;
    int sg;
    if (r < segs.n_out[0]) {
        sg = 0;
    } else if (segs.n > 1 && r < segs.n_out[0] + segs.n_out[1]) {
        sg = 1;
        r -= segs.n_out[0];
    } else if (segs.n > 2 && r < segs.n_out[0] + segs.n_out[1] + segs.n_out[2]) {
        sg = 2;
        r -= segs.n_out[0] + segs.n_out[1];
    } else {
        return;
    }
    const int dt = sg == 0 ? segs.dtype[0] : sg == 1 ? segs.dtype[1] : segs.dtype[2];
    const uint8_t* wbase = sg == 0 ? segs.w[0] : sg == 1 ? segs.w[1] : segs.w[2];
    const size_t rb = sg == 0 ? segs.row_bytes[0] : sg == 1 ? segs.row_bytes[1] : segs.row_bytes[2];
    float* ybase = sg == 0 ? segs.y[0] : sg == 1 ? segs.y[1] : segs.y[2];
    const uint8_t* row = wbase + r * rb;
    float acc;
    if (dt == kGgmlQ4K || dt == kGgmlQ6K) {
        acc = -0.0f;
        constexpr int kU = 4;
        for (size_t b0 = 0; b0 < nb; b0 += kU) {
            if (dt == kGgmlQ4K) {
                Q4Ld L[kU];
#pragma unroll
                for (int u = 0; u < kU; ++u)
                    if (b0 + u < nb)
                        L[u] = load_q4k(row + (b0 + u) * 144, s_q + (b0 + u) * kQK, s_sc[b0 + u], s_sum + (b0 + u) * 8, lane);
#pragma unroll
                for (int u = 0; u < kU; ++u)
                    if (b0 + u < nb) acc = __fadd_rn(acc, dot_q4k(L[u], lane));
            } else {
                Q6Ld L[kU];
#pragma unroll
                for (int u = 0; u < kU; ++u)
                    if (b0 + u < nb) L[u] = load_q6k(row + (b0 + u) * 210, s_q + (b0 + u) * kQK, s_sc[b0 + u], lane);
#pragma unroll
                for (int u = 0; u < kU; ++u)
                    if (b0 + u < nb) acc = __fadd_rn(acc, dot_q6k(L[u], lane));
            }
        }
    } else {
        acc = dt == kGgmlF32 ? row_dot<kGgmlF32>(row, x, n_in, lane) : row_dot<kGgmlF16>(row, x, n_in, lane);
    }
    if (lane == 0) ybase[r] = acc;
}

// One token, K-quant weights only: one LANE per 256-weight block. A row's nb blocks sit on
// nb lanes (L = nb rounded up to a power of two lanes per row, 32/L rows per warp); each lane
// forms its block's exact integer dot alone (64 dp4a, no cross-lane reduction) and the f32
// block value as qmatmul_kernel does, then the row's values are added in block order through
// shuffles. Same bits as qmatmul_kernel, with ~30x fewer instructions per block.
constexpr int kQStride = 272;  // Q8 activations of a block in shared memory, padded against bank conflicts

__device__ __forceinline__ float lane_block_q4k(const uint8_t* blk, const int8_t* qx, float sx, const int* sums) {
    const uint4* p = reinterpret_cast<const uint4*>(blk);
    const uint4 head = p[0];
    int sd = 0, sm = 0;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        int sc0, m0, sc1, m1;
        scale_min_head(2 * c, head, sc0, m0);
        scale_min_head(2 * c + 1, head, sc1, m1);
        sm += m0 * sums[2 * c] + m1 * sums[2 * c + 1];
        const uint4 q0 = p[1 + 2 * c], q1 = p[2 + 2 * c];
        const uint32_t qw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
        const int4* xl = reinterpret_cast<const int4*>(qx + (2 * c) * 32);
        const int4* xh = reinterpret_cast<const int4*>(qx + (2 * c + 1) * 32);
        const int4 a0 = xl[0], a1 = xl[1], b0 = xh[0], b1 = xh[1];
        const int xa[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        const int xb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
        int lo = 0, hi = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            lo = __dp4a((int)(qw[i] & 0x0f0f0f0fu), xa[i], lo);
            hi = __dp4a((int)((qw[i] >> 4) & 0x0f0f0f0fu), xb[i], hi);
        }
        sd += sc0 * lo + sc1 * hi;
    }
    const float d = f16_bits_to_f32(head.x & 0xffffu), dmin = f16_bits_to_f32(head.x >> 16);
    return __fmul_rn(sx, __fsub_rn(__fmul_rn(d, __int2float_rn(sd)), __fmul_rn(dmin, __int2float_rn(sm))));
}

// 16 bytes from a 2-byte-aligned address, as four little-endian words
__device__ __forceinline__ void ld16_a2(const uint8_t* p, uint32_t* w) {
    const uint16_t* h = reinterpret_cast<const uint16_t*>(p);
#pragma unroll
    for (int i = 0; i < 4; ++i) w[i] = (uint32_t)h[2 * i] | ((uint32_t)h[2 * i + 1] << 16);
}

// sums16: the 16-wide sub-block sums of qx, so that Σ (q - 32) x = Σ q x - 32 Σ x (exact): the
// 6-bit q (0..63, a non-negative s8) goes into dp4a as it is
__device__ __forceinline__ float lane_block_q6k(const uint8_t* blk, const int8_t* qx, float sx, const int* sums16) {
    uint32_t scw[4];
    ld16_a2(blk + 192, scw);
    int s = 0;
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
        for (int sub = 0; sub < 2; ++sub) {
            uint32_t lo[4], hi[4], qh[4];
            ld16_a2(blk + n * 64 + sub * 16, lo);       // ql[0..32) part: groups 0 (low) and 2 (high)
            ld16_a2(blk + n * 64 + 32 + sub * 16, hi);  // ql[32..64) part: groups 1 and 3
            ld16_a2(blk + 128 + n * 32 + sub * 16, qh);
#pragma unroll
            for (int g = 0; g < 4; ++g) {
                const int k = n * 8 + 2 * g + sub;
                const int4 xv = *reinterpret_cast<const int4*>(qx + k * 16);
                const int xw[4] = {xv.x, xv.y, xv.z, xv.w};
                int t = 0;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const uint32_t src = (g & 1) ? hi[i] : lo[i];
                    const uint32_t nib = (g >= 2 ? src >> 4 : src) & 0x0f0f0f0fu;
                    // the 2-bit field (qh >> 2g) & 3, moved to bits 4-5 of each byte
                    const uint32_t hq = g == 0 ? qh[i] << 4 : g == 1 ? qh[i] << 2 : g == 2 ? qh[i] : qh[i] >> 2;
                    t = __dp4a((int)(nib | (hq & 0x30303030u)), xw[i], t);  // bytes q in [0, 63]
                }
                const int sc = (int)(int8_t)((scw[k >> 2] >> (8 * (k & 3))) & 0xffu);
                s += (t - 32 * sums16[k]) * sc;
            }
        }
    const float d = f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(blk + 208));
    return __fmul_rn(sx, __fmul_rn(d, __int2float_rn(s)));
}

// Q8 of x [nb blocks] into shared memory (as quantize_q8_kernel: same bits), one warp per block;
// a block's quants at stride kQStride
__device__ __forceinline__ void q8_into_smem(const float* x, int nb, int8_t* s_q, float* s_sc, int* s_sum,
                                             int* s_sum16) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, n_warps = blockDim.x >> 5;
    for (int blk = warp; blk < nb; blk += n_warps) {  // Q8 of x, as quantize_q8_kernel
        const float* xb = x + (size_t)blk * kQK + lane * 8;
        const float4 a = *reinterpret_cast<const float4*>(xb), b = *reinterpret_cast<const float4*>(xb + 4);
        const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
        float amax = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        const float inv = amax > 0.f ? __fdiv_rn(127.0f, amax) : 0.f;
        int8_t qv[8];
        int sm = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            float r = roundf(__fmul_rn(v[i], inv));
            r = fminf(fmaxf(r, -127.f), 127.f);
            qv[i] = (int8_t)r;
            sm += qv[i];
        }
        *reinterpret_cast<uint2*>(s_q + blk * kQStride + lane * 8) = *reinterpret_cast<const uint2*>(qv);
        sm += __shfl_xor_sync(0xffffffffu, sm, 1);  // a 16-wide sub-block is 2 lanes
        if ((lane & 1) == 0) s_sum16[blk * 16 + (lane >> 1)] = sm;
        sm += __shfl_xor_sync(0xffffffffu, sm, 2);
        if ((lane & 3) == 0) s_sum[blk * 8 + (lane >> 2)] = sm;
        if (lane == 0) s_sc[blk] = __fdiv_rn(amax, 127.0f);
    }
}

__global__ void __launch_bounds__(256) qmv_lane_kernel(QmvSegs segs, const float* x, size_t n_in) {
    __shared__ __align__(16) int8_t s_q[(kMvMaxIn / kQK) * kQStride];
    __shared__ float s_sc[kMvMaxIn / kQK];
    __shared__ int s_sum[kMvMaxIn / 32];
    __shared__ int s_sum16[kMvMaxIn / 16];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nb = (int)(n_in / kQK);
    q8_into_smem(x, nb, s_q, s_sc, s_sum, s_sum16);
    __syncthreads();
    int L = 1;
    while (L < nb) L <<= 1;
    const int b = lane & (L - 1);
    size_t r = ((size_t)blockIdx.x * 8 + warp) * (32 / L) + lane / L;
    int sg = -1;
    if (r < segs.n_out[0]) {
        sg = 0;
    } else if (segs.n > 1 && r < segs.n_out[0] + segs.n_out[1]) {
        sg = 1;
        r -= segs.n_out[0];
    } else if (segs.n > 2 && r < segs.n_out[0] + segs.n_out[1] + segs.n_out[2]) {
        sg = 2;
        r -= segs.n_out[0] + segs.n_out[1];
    }
    float v = 0.f;
    if (sg >= 0 && b < nb) {
        const int dt = sg == 0 ? segs.dtype[0] : sg == 1 ? segs.dtype[1] : segs.dtype[2];
        const uint8_t* wb = sg == 0 ? segs.w[0] : sg == 1 ? segs.w[1] : segs.w[2];
        const size_t rb = sg == 0 ? segs.row_bytes[0] : sg == 1 ? segs.row_bytes[1] : segs.row_bytes[2];
        const uint8_t* row = wb + r * rb;
        v = dt == kGgmlQ4K ? lane_block_q4k(row + (size_t)b * 144, s_q + b * kQStride, s_sc[b], s_sum + b * 8)
                           : lane_block_q6k(row + (size_t)b * 210, s_q + b * kQStride, s_sc[b], s_sum16 + b * 16);
    }
    const int base = lane & ~(L - 1);
    float acc = -0.0f;  // the blocks of the row, added in order
    for (int j = 0; j < nb; ++j) acc = __fadd_rn(acc, __shfl_sync(0xffffffffu, v, base + j));
    if (sg >= 0 && b == 0) {
        float* yb = sg == 0 ? segs.y[0] : sg == 1 ? segs.y[1] : segs.y[2];
        yb[r] = acc;
    }
}

// A Q6_K block at a 2-byte aligned shared-memory address whose offset mod 16 is the same for
// the whole warp: 14 aligned 16-byte loads, realigned in registers (warp-uniform selects and a
// funnel shift), then lane_block_q6k's arithmetic on the words (same integer sums).
__device__ __forceinline__ float q6k_block_realigned(const unsigned char* blk, const int8_t* qx, float sx,
                                                     const int* sums16) {
    const int o = (int)(reinterpret_cast<uintptr_t>(blk) & 15);
    const uint4* p = reinterpret_cast<const uint4*>(blk - o);
    uint32_t v[59];
#pragma unroll
    for (int i = 0; i < 14; ++i) {
        const uint4 t = p[i];
        v[4 * i] = t.x, v[4 * i + 1] = t.y, v[4 * i + 2] = t.z, v[4 * i + 3] = t.w;
    }
    v[56] = v[57] = v[58] = 0;
    const int ws = o >> 2;
    const uint32_t bs = (uint32_t)(o & 3) * 8;
#pragma unroll
    for (int i = 0; i < 57; ++i) v[i] = (ws & 2) ? v[i + 2] : v[i];
#pragma unroll
    for (int i = 0; i < 56; ++i) v[i] = (ws & 1) ? v[i + 1] : v[i];
    uint32_t w[53];  // ql: 0..31, qh: 32..47, scales: 48..51, d: low half of 52
#pragma unroll
    for (int i = 0; i < 53; ++i) w[i] = __funnelshift_r(v[i], v[i + 1], bs);
    int s = 0;
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
        for (int sub = 0; sub < 2; ++sub)
#pragma unroll
            for (int g = 0; g < 4; ++g) {
                const int k = n * 8 + 2 * g + sub;
                const int4 xv = *reinterpret_cast<const int4*>(qx + k * 16);
                const int xw[4] = {xv.x, xv.y, xv.z, xv.w};
                int t = 0;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const uint32_t src = w[n * 16 + (g & 1) * 8 + sub * 4 + i];
                    const uint32_t qh = w[32 + n * 8 + sub * 4 + i];
                    const uint32_t nib = (g >= 2 ? src >> 4 : src) & 0x0f0f0f0fu;
                    const uint32_t hq = g == 0 ? qh << 4 : g == 1 ? qh << 2 : g == 2 ? qh : qh >> 2;
                    t = __dp4a((int)(nib | (hq & 0x30303030u)), xw[i], t);
                }
                const int sc = (int)(int8_t)((w[48 + (k >> 2)] >> (8 * (k & 3))) & 0xffu);
                s += (t - 32 * sums16[k]) * sc;
            }
    const float d = f16_bits_to_f32(w[52] & 0xffffu);
    return __fmul_rn(sx, __fmul_rn(d, __int2float_rn(s)));
}

// One token against a large matrix (the vocab-sized logits head): persistent CTAs, each
// quantizing x once and streaming its chunks of 256 blocks (rows * row_bytes, contiguous) into
// a 3-slot shared-memory ring with 1-D bulk copies (cp.async.bulk, mbarrier complete_tx), so
// each SM keeps ~100 KB of weights in flight. The arithmetic is qmv_lane_kernel's (one lane
// per block, the row's block values added in order): same bits. Waits are bounded; on timeout
// the CTA stores kErrWaitTimeout to *err, waits (bounded) for its copies in flight, returns.
constexpr int kStreamStages = 3;
constexpr int kStreamChunkMax = 256 * 210;
constexpr int kStreamThreads = 512;  // two groups of 8 warps

__device__ __forceinline__ bool stream_wait(uint32_t bar, unsigned parity) {
    for (long long it = 0; it < (1ll << 22); ++it) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(bar), "r"(parity)
            : "memory");
        if (ok) return true;
    }
    return false;
}

// The logits head variant (kHead) also does the final RMSNorm of x and the greedy argmax:
// every CTA normalizes x itself with rmsnorm_row_kernel's arithmetic and reduction tree (a
// 1024-wide tree of f64 partial sums, evaluated by 256 threads four virtual threads each), so
// the normalized x has the same bits; each CTA keeps the first index of its rows' maximum
// (strict `>` in increasing row order, NaN never wins) and the last CTA to finish reduces the
// CTAs' candidates to the token (ties to the lower index) and re-arms the counter.
struct HeadArgs {
    const float* gain = nullptr;
    float eps = 0.f;
    float* cand_v = nullptr;  // [gridDim.x]
    uint32_t* cand_i = nullptr;
    unsigned* counter = nullptr;  // 0 between calls
    uint32_t* token = nullptr;    // nullable
};

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ void better_of(float& v, uint32_t& i, float ov, uint32_t oi) {
    if (oi == 0xffffffffu) return;
    if (i == 0xffffffffu || ov > v || (ov == v && oi < i)) v = ov, i = oi;
}

template <bool kHead>
__global__ void __launch_bounds__(kStreamThreads, 1)
    qmv_stream_kernel(int dtype, const uint8_t* w, size_t rb, size_t n_out, const float* x, size_t n_in,
                      int rows_per_chunk, float* y, int* err, HeadArgs ha) {
    extern __shared__ __align__(128) unsigned char ring[];
    __shared__ __align__(16) int8_t s_q[(kMvMaxIn / kQK) * kQStride];
    __shared__ float s_sc[kMvMaxIn / kQK];
    __shared__ int s_sum[kMvMaxIn / 32];
    __shared__ int s_sum16[kMvMaxIn / 16];
    __shared__ int s_fail[2];
    // the chunk last issued into each ring slot: a group waits for its chunk to be issued before
    // it waits on the slot's mbarrier, so it never tests a phase parity one phase early (the
    // other group may still hold the slot's previous chunk)
    __shared__ long long s_issued[kStreamStages];
    __shared__ __align__(16) float s_x[kHead ? kMvMaxIn : 1];
    __shared__ double s_part[32];
    __shared__ float s_bv[kStreamThreads / 32];
    __shared__ uint32_t s_bi[kStreamThreads / 32];
    __shared__ bool s_last;
    __shared__ float s_v[2][32 * 9];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // two groups of 8 warps take alternate chunks of the ring (group g: chunks k = g, g + 2, ...)
    const int grp = warp >> 3, gw = warp & 7, gtid = tid & 255;
    const int nb = (int)(n_in / kQK);
    const uint32_t ring_s = (uint32_t)__cvta_generic_to_shared(ring);
    const uint32_t bar0 = ring_s + kStreamStages * kStreamChunkMax;
    const size_t n_chunks = (n_out + rows_per_chunk - 1) / rows_per_chunk;
    auto issue = [&](size_t k) {  // by one thread: chunk k of this CTA into ring slot k % 3
        const size_t c = blockIdx.x + k * gridDim.x;
        if (c >= n_chunks) return;
        const size_t r0 = c * rows_per_chunk;
        const uint32_t bytes = (uint32_t)(std::min<size_t>(rows_per_chunk, n_out - r0) * rb);
        const uint32_t bar = bar0 + 8 * (uint32_t)(k % kStreamStages);
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
        asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                         ring_s + (uint32_t)(k % kStreamStages) * kStreamChunkMax),
                     "l"(w + r0 * rb), "r"(bytes), "r"(bar)
                     : "memory");
        __threadfence_block();  // the expect_tx before the record
        reinterpret_cast<volatile long long*>(s_issued)[k % kStreamStages] = (long long)k;
    };
    auto issued_wait = [&](size_t k) {  // bounded
        for (long long it = 0; it < (1ll << 22); ++it)
            if (reinterpret_cast<volatile long long*>(s_issued)[k % kStreamStages] == (long long)k) return true;
        return false;
    };
    auto group_sync = [&]() { asm volatile("bar.sync %0, 256;" ::"r"(1 + grp) : "memory"); };
    if (tid == 0) {
        for (int i = 0; i < kStreamStages; ++i) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar0 + 8 * i));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        s_fail[0] = s_fail[1] = 0;
        for (int k = 0; k < kStreamStages; ++k) s_issued[k] = -1;
        for (int k = 0; k < kStreamStages; ++k) issue(k);
    }
    if constexpr (kHead) {  // x <- rmsnorm(x, gain, eps) in shared memory
        const int n = (int)n_in;
        double ss[2];
#pragma unroll
        for (int j = 0; j < 2; ++j) {  // virtual thread tid + 512 j of the 1024-wide tree
            double acc = 0.0;
            for (int i = tid + kStreamThreads * j; i < n; i += 1024) acc += (double)__fmul_rn(x[i], x[i]);
            ss[j] = warp_sum_d(acc);
        }
        if (lane == 0) s_part[warp] = ss[0], s_part[warp + 16] = ss[1];
        __syncthreads();
        if (warp == 0) {
            const double v = warp_sum_d(s_part[lane]);
            if (lane == 0) {
                const float mean = __double2float_rn(v / (double)n);
                s_part[0] = (double)__fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, ha.eps)));
            }
        }
        __syncthreads();
        const float scale = (float)s_part[0];
        for (int i = tid; i < n; i += kStreamThreads) s_x[i] = __fmul_rn(__fmul_rn(x[i], scale), ha.gain[i]);
        __syncthreads();
        q8_into_smem(s_x, nb, s_q, s_sc, s_sum, s_sum16);
    } else {
        q8_into_smem(x, nb, s_q, s_sc, s_sum, s_sum16);
    }
    __syncthreads();
    int L = 1;
    while (L < nb) L <<= 1;
    const int b = lane & (L - 1), rloc = gw * (32 / L) + lane / L, base = lane & ~(L - 1);
    const int bbytes = dtype == kGgmlQ4K ? 144 : 210;
    float best_v = 0.f;
    uint32_t best_i = 0xffffffffu;
    // Q6_K blocks sit at 2-byte offsets: with at most 8 blocks a row, a warp takes one block
    // column of 32 rows, so its lanes share the block's offset mod 16 (aligned loads, no conflicts
    // at the row stride), and the group's warp 0 adds each row's block values in order
    const bool q6_cols = dtype == kGgmlQ6K && rows_per_chunk == 32 && nb <= 8;
    size_t k = grp;
    for (; blockIdx.x + k * gridDim.x < n_chunks; k += 2) {
        const uint32_t bar = bar0 + 8 * (uint32_t)(k % kStreamStages);
        const unsigned parity = (unsigned)((k / kStreamStages) & 1);
        if (gtid == 0 && !(issued_wait(k) && stream_wait(bar, parity))) s_fail[grp] = 1;
        group_sync();
        if (*reinterpret_cast<volatile int*>(&s_fail[grp])) break;  // written only before the barrier
        stream_wait(bar, parity);  // this thread's own acquire of the landed bytes (succeeds at once)
        const size_t c0 = (blockIdx.x + k * gridDim.x) * rows_per_chunk;
        const unsigned char* slot = ring + (k % kStreamStages) * kStreamChunkMax;
        size_t r;
        float acc = -0.0f;  // the blocks of the row, added in order
        bool mine;
        if (q6_cols) {  // warp = block column, lane = row (32 rows per chunk)
            r = c0 + lane;
            if (gw < nb && r < n_out)
                s_v[grp][lane * 9 + gw] = q6k_block_realigned(slot + (size_t)lane * rb + (size_t)gw * 210,
                                                               s_q + gw * kQStride, s_sc[gw], s_sum16 + gw * 16);
            group_sync();
            mine = gw == 0 && r < n_out;
            if (mine)
                for (int j = 0; j < nb; ++j) acc = __fadd_rn(acc, s_v[grp][lane * 9 + j]);
        } else {
            r = c0 + rloc;
            const unsigned char* row = slot + (size_t)rloc * rb;
            float v = 0.f;
            if (r < n_out && b < nb && rloc < rows_per_chunk)
                v = dtype == kGgmlQ4K
                        ? lane_block_q4k(row + (size_t)b * bbytes, s_q + b * kQStride, s_sc[b], s_sum + b * 8)
                        : lane_block_q6k(row + (size_t)b * bbytes, s_q + b * kQStride, s_sc[b], s_sum16 + b * 16);
            for (int j = 0; j < nb; ++j) acc = __fadd_rn(acc, __shfl_sync(0xffffffffu, v, base + j));
            mine = r < n_out && b == 0 && rloc < rows_per_chunk;
        }
        if (mine) {
            y[r] = acc;
            if constexpr (kHead)
                if (acc > -CUDART_INF_F && (best_i == 0xffffffffu || acc > best_v)) best_v = acc, best_i = (uint32_t)r;
        }
        group_sync();  // the slot is consumed
        if (gtid == 0) issue(k + kStreamStages);
    }
    if (gtid == 0 && s_fail[grp]) {
        *reinterpret_cast<volatile int*>(err) = kErrWaitTimeout;
        // copies still in flight must land before the CTA exits: of the chunks this group may
        // have left unconsumed (k, and the refill k + 1 it issued), those that were issued
        for (size_t i = k; i < k + 2; ++i)
            if (blockIdx.x + i * gridDim.x < n_chunks &&
                reinterpret_cast<volatile long long*>(s_issued)[i % kStreamStages] == (long long)i)
                stream_wait(bar0 + 8 * (uint32_t)(i % kStreamStages), (unsigned)((i / kStreamStages) & 1));
    }
    __syncthreads();
    if constexpr (kHead) {
        // a CTA whose wait gave up still takes part (with what it has), so the counter is
        // re-armed; the error word marks the result invalid
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
            better_of(best_v, best_i, __shfl_xor_sync(0xffffffffu, best_v, o), __shfl_xor_sync(0xffffffffu, best_i, o));
        if (lane == 0) s_bv[warp] = best_v, s_bi[warp] = best_i;
        __syncthreads();
        if (tid == 0) {
            for (int i = 1; i < kStreamThreads / 32; ++i) better_of(s_bv[0], s_bi[0], s_bv[i], s_bi[i]);
            ha.cand_v[blockIdx.x] = s_bv[0];
            ha.cand_i[blockIdx.x] = s_bi[0];
            __threadfence();
            s_last = atomicAdd(ha.counter, 1u) == gridDim.x - 1;
        }
        __syncthreads();
        if (s_last && warp == 0) {  // the last CTA: every candidate is written (fence + counter)
            __threadfence();
            float v = 0.f;
            uint32_t i = 0xffffffffu;
            for (unsigned c = lane; c < gridDim.x; c += 32)
                better_of(v, i, reinterpret_cast<volatile float*>(ha.cand_v)[c],
                          reinterpret_cast<volatile uint32_t*>(ha.cand_i)[c]);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1)
                better_of(v, i, __shfl_xor_sync(0xffffffffu, v, o), __shfl_xor_sync(0xffffffffu, i, o));
            if (lane == 0) {
                if (ha.token) *ha.token = i == 0xffffffffu ? 0u : i;
                *ha.counter = 0;  // re-armed for the next call (or graph replay)
            }
        }
    }
}

__global__ void dequant_kernel(int dtype, const uint8_t* data, size_t n, float* out) {
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        float v;
        if (dtype == kGgmlF32) {
            v = reinterpret_cast<const float*>(data)[i];
        } else if (dtype == kGgmlF16) {
            v = ld_f16(data + 2 * i);
        } else if (dtype == kGgmlQ4K) {
            const uint8_t* b = data + (i / kQK) * 144;
            const int e = (int)(i % kQK), chunk = e / 64, hi = (e % 64) / 32, l = e % 32;
            int sc, m;
            scale_min_k4(2 * chunk + hi, b + 4, sc, m);
            const uint8_t q = b[16 + chunk * 32 + l];
            const float d = ld_f16(b), dmin = ld_f16(b + 2);
            v = __fsub_rn(__fmul_rn(__fmul_rn(d, (float)sc), (float)(hi ? q >> 4 : q & 0x0f)),
                          __fmul_rn(dmin, (float)m));
        } else {  // Q6_K
            const uint8_t* b = data + (i / kQK) * 210;
            const int e = (int)(i % kQK), nh = e / 128, r = e % 128, grp = r / 32, l = r % 32;
            const uint8_t* ql = b + nh * 64;
            const uint8_t* qh = b + 128 + nh * 32;
            const int8_t* sc = reinterpret_cast<const int8_t*>(b + 192 + nh * 8);
            const int lb = (grp & 1) ? ql[l + 32] : ql[l];
            const int low = grp >= 2 ? lb >> 4 : lb & 0x0f;
            const int q = (low | (((qh[l] >> (2 * grp)) & 3) << 4)) - 32;
            v = __fmul_rn(__fmul_rn(ld_f16(b + 208), (float)sc[l / 16 + 2 * grp]), (float)q);
        }
        out[i] = v;
    }
}

}  // namespace

size_t ggml_row_bytes(int dtype, size_t n_in) {
    switch (dtype) {
        case kGgmlF32: return 4 * n_in;
        case kGgmlF16: return 2 * n_in;
        case kGgmlQ4K: return n_in / kQK * 144;
        case kGgmlQ6K: return n_in / kQK * 210;
        default: return 0;
    }
}

bool kquant_tc_enabled() {
    static const bool on = [] {
        const char* e = getenv("BEBELM_QMM_TC");
        return !(e && e[0] == '0');
    }();
    return on;
}

cudaError_t launch_quantize_q8(const float* x, size_t n_in, size_t n_tokens, int8_t* q, float* scales, int* sums,
                               cudaStream_t s) {
    const size_t blocks = n_in / kQK * n_tokens;
    if (blocks == 0) return cudaSuccess;
    quantize_q8_kernel<<<(unsigned)((blocks + 7) / 8), 256, 0, s>>>(x, n_in, q, scales, sums, blocks);
    return cudaGetLastError();
}

cudaError_t launch_qmatmul(int dtype, const uint8_t* w, size_t n_in, size_t n_out, const float* x, size_t n_tokens,
                           const int8_t* q8, const float* q8_scales, const int* q8_sums, float* y, int* err,
                           cudaStream_t s) {
    if (n_out == 0 || n_tokens == 0) return cudaSuccess;
    const size_t rb = ggml_row_bytes(dtype, n_in);
    if ((dtype == kGgmlQ4K || dtype == kGgmlQ6K) && n_tokens >= kTcMinTokens && err && kquant_tc_enabled()) {
        const cudaError_t e = launch_kquant_tc(dtype, w, n_in, n_out, n_tokens, q8, q8_scales, q8_sums, y, err, s);
        if (e != cudaErrorNotSupported) return e;  // else: no tensor maps for these buffers; dp4a below
    }
    if ((dtype == kGgmlQ4K || dtype == kGgmlQ6K) && n_tokens >= kTiledMinTokens) {
        const dim3 tg((unsigned)((n_out + kTR - 1) / kTR), (unsigned)((n_tokens + kTT - 1) / kTT));
        static bool attr_set[64][2] = {};
        int dev = 0;
        cudaGetDevice(&dev);
        const int which = dtype == kGgmlQ4K ? 0 : 1;
        if (dev < 0 || dev >= 64 || !attr_set[dev][which]) {
            cudaError_t e = which == 0 ? cudaFuncSetAttribute(qmatmul_tiled_kernel<kGgmlQ4K>,
                                                              cudaFuncAttributeMaxDynamicSharedMemorySize, kTiledDynBytes)
                                       : cudaFuncSetAttribute(qmatmul_tiled_kernel<kGgmlQ6K>,
                                                              cudaFuncAttributeMaxDynamicSharedMemorySize, kTiledDynBytes);
            if (e != cudaSuccess) return e;
            if (dev >= 0 && dev < 64) attr_set[dev][which] = true;
        }
        if (dtype == kGgmlQ4K)
            qmatmul_tiled_kernel<kGgmlQ4K><<<tg, 256, kTiledDynBytes, s>>>(w, rb, n_in, n_out, n_tokens, q8, q8_scales,
                                                                          q8_sums, y);
        else
            qmatmul_tiled_kernel<kGgmlQ6K><<<tg, 256, kTiledDynBytes, s>>>(w, rb, n_in, n_out, n_tokens, q8, q8_scales,
                                                                          q8_sums, y);
        return cudaGetLastError();
    }
    const dim3 grid((unsigned)((n_out + 7) / 8), (unsigned)n_tokens);
    switch (dtype) {
        case kGgmlF32: qmatmul_kernel<kGgmlF32><<<grid, 256, 0, s>>>(w, rb, n_in, n_out, x, q8, q8_scales, q8_sums, y); break;
        case kGgmlF16: qmatmul_kernel<kGgmlF16><<<grid, 256, 0, s>>>(w, rb, n_in, n_out, x, q8, q8_scales, q8_sums, y); break;
        case kGgmlQ4K: qmatmul_kernel<kGgmlQ4K><<<grid, 256, 0, s>>>(w, rb, n_in, n_out, x, q8, q8_scales, q8_sums, y); break;
        case kGgmlQ6K: qmatmul_kernel<kGgmlQ6K><<<grid, 256, 0, s>>>(w, rb, n_in, n_out, x, q8, q8_scales, q8_sums, y); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_qmv_multi(const QmvSegs& segs, const float* x, size_t n_in, cudaStream_t s) {
    if (n_in > (size_t)kMvMaxIn || segs.n < 1 || segs.n > 3) return cudaErrorInvalidValue;
    size_t rows = 0;
    for (int i = 0; i < segs.n; ++i) rows += segs.n_out[i];
    if (rows == 0) return cudaSuccess;
    bool kq = true;
    for (int i = 0; i < segs.n; ++i) kq &= segs.dtype[i] == kGgmlQ4K || segs.dtype[i] == kGgmlQ6K;
    if (kq && n_in % kQK == 0) {
        size_t L = 1;
        while (L < n_in / kQK) L <<= 1;
        const size_t rows_per_cta = 8 * (32 / L);
        qmv_lane_kernel<<<(unsigned)((rows + rows_per_cta - 1) / rows_per_cta), 256, 0, s>>>(segs, x, n_in);
    } else {
        qmv_multi_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, s>>>(segs, x, n_in);
    }
    return cudaGetLastError();
}

static cudaError_t qmv_stream_impl(int dtype, const uint8_t* w, size_t n_out, const float* x, size_t n_in, float* y,
                                   int* err, cudaStream_t s, const HeadArgs* head) {
    if ((dtype != kGgmlQ4K && dtype != kGgmlQ6K) || n_in % kQK || n_in > (size_t)kMvMaxIn || n_out == 0 || !err)
        return cudaErrorNotSupported;
    const size_t rb = ggml_row_bytes(dtype, n_in);
    if ((rb & 15) || (reinterpret_cast<uintptr_t>(w) & 15)) return cudaErrorNotSupported;
    int L = 1;
    while ((size_t)L < n_in / kQK) L <<= 1;
    const int rows_per_chunk = 8 * (32 / L);
    if ((size_t)rows_per_chunk * rb > (size_t)kStreamChunkMax) return cudaErrorNotSupported;
    static int n_sm[64] = {};
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorNotSupported;
    const int dyn = kStreamStages * kStreamChunkMax + 64;
    if (!attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(qmv_stream_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(qmv_stream_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn);
        if (e != cudaSuccess) return e;
        e = cudaDeviceGetAttribute(&n_sm[dev], cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return e;
        attr_set[dev] = true;
    }
    const size_t n_chunks = (n_out + rows_per_chunk - 1) / rows_per_chunk;
    const unsigned grid = (unsigned)std::min<size_t>(n_chunks, (size_t)n_sm[dev]);
    if (head)
        qmv_stream_kernel<true><<<grid, kStreamThreads, dyn, s>>>(dtype, w, rb, n_out, x, n_in, rows_per_chunk, y, err, *head);
    else
        qmv_stream_kernel<false><<<grid, kStreamThreads, dyn, s>>>(dtype, w, rb, n_out, x, n_in, rows_per_chunk, y, err, HeadArgs{});
    return cudaGetLastError();
}

cudaError_t launch_qmv_stream(int dtype, const uint8_t* w, size_t n_out, const float* x, size_t n_in, float* y,
                              int* err, cudaStream_t s) {
    return qmv_stream_impl(dtype, w, n_out, x, n_in, y, err, s, nullptr);
}

cudaError_t launch_head_stream(int dtype, const uint8_t* w, size_t vocab, const float* h, const float* gain, float eps,
                               size_t hidden, float* logits, uint32_t* token, float* cand_v, uint32_t* cand_i,
                               unsigned* counter, int* err, cudaStream_t s) {
    HeadArgs ha;
    ha.gain = gain;
    ha.eps = eps;
    ha.cand_v = cand_v;
    ha.cand_i = cand_i;
    ha.counter = counter;
    ha.token = token;
    return qmv_stream_impl(dtype, w, vocab, h, hidden, logits, err, s, &ha);
}

cudaError_t launch_dequantize(int dtype, const uint8_t* data, size_t n, float* out, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    const size_t blocks = std::min<size_t>((n + 255) / 256, 148 * 16);
    dequant_kernel<<<(unsigned)blocks, 256, 0, s>>>(dtype, data, n, out);
    return cudaGetLastError();
}

}  // namespace bebelm
