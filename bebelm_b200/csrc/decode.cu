// Kernel 3: split-K single-query GQA decode over the paged KV cache, with the
// combine of the splits fused into the last CTA of each (sequence, kv head).
//
// Computes, for every query head h of kv head g = h / group (the reference's
// `attention_decode`, src/kernels/attention.rs:17-55):
//   out[h] = Σ_j softmax_j(q[h]·k[j,g] * scale) · v[j,g]
// as an online (flash-decoding) softmax in fp32: each CTA streams a run of
// whole KV pages for one kv head, keeps the running max / sum / weighted V of
// up to 4 query heads of that group (so every K/V byte is read from HBM once,
// not once per query head as the reference does), and writes a partial
// (max, sum, acc[64]) per head. The last CTA to finish a (sequence, kv head)
// merges all partials and writes the output.
//
// Data movement: one thread issues 1-D bulk TMA copies (cp.async.bulk) of a
// page's K rows (16 KB) and V rows (16 KB) for this kv head into a 3-stage
// shared-memory ring, completed on an mbarrier; 2 CTAs per SM keep ~4 pages
// (128 KB) in flight per SM. Every wait is bounded: on timeout the CTA records
// kErrWaitTimeout, drains its own copies (bounded again) and returns.
//
// Compute mapping (128 threads, 4 warps): warp w owns rows 16w..16w+15 of each
// 64-row page; lane = 4*j + p handles rows 16w+j and 16w+8+j and the 16 dims
// of float4 chunks c_i = ((i+j)&3)*4 + p, i = 0..3. The rotation by j makes
// every float4 shared-memory read conflict-free and lets each lane keep its q
// slice in registers; the 4 lanes of a row reduce the dot with two xor
// shuffles (identical result on all 4 lanes).
#include "internal.h"

namespace bebelm {
namespace {

constexpr int kStages = 3;
constexpr int kThreads = 128;
constexpr int kStageBytes = 2 * kPageRowFloats * 4;  // K + V rows of one page, one kv head
constexpr long long kWaitLimit = 1ll << 22;          // try_wait polls before giving up

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, unsigned parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, unsigned parity) {
    for (long long it = 0; it < kWaitLimit; ++it)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, unsigned bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ float fast_exp2(float x) { return exp2f(x); }

template <int HPC>
__global__ void __launch_bounds__(kThreads, 2) decode_kernel(DecodeArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    float* stages = reinterpret_cast<float*>(smem);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
    __shared__ float s_m[4][HPC], s_l[4][HPC];
    __shared__ int s_last;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int j = lane >> 2, p = lane & 3;
    const int NY = a.n_kv * a.n_sub;
    const int y = blockIdx.y;
    const int kvh = y / a.n_sub, sub = y % a.n_sub;
    const int h0 = kvh * a.group + sub * HPC;

    // which sequence owns this split
    const int gsplit = blockIdx.x;
    int lo = 0, hi = a.n_seqs - 1;
    while (lo < hi) {
        int mid = (lo + hi + 1) >> 1;
        if (a.seqs[mid].split0 <= gsplit) lo = mid; else hi = mid - 1;
    }
    const int seq = lo;
    const DecodeSeq S = a.n_seqs == 1 ? a.one : a.seqs[seq];
    const int split = gsplit - S.split0;
    const long long first_page = S.base >> 6;
    const long long last_page = S.len > 0 ? (S.base + S.len - 1) >> 6 : first_page - 1;
    const long long p0 = first_page + (long long)split * a.pages_per_split;
    long long p1 = p0 + a.pages_per_split;
    if (p1 > last_page + 1) p1 = last_page + 1;
    const int np = p1 > p0 ? (int)(p1 - p0) : 0;

    auto issue = [&](int i) {
        const int st = i % kStages;
        const long long lp = p0 + i;
        const int phys = S.table[(int)(lp % S.cap)];
        const float* kp = a.pv.base + (size_t)phys * a.pv.page_floats + a.pv.layer_off +
                          (size_t)kvh * kPageRowFloats;
        const float* vp = kp + a.pv.block_floats;
        float* dk = stages + (size_t)st * (2 * kPageRowFloats);
        mbar_expect_tx(&full[st], kStageBytes);
        bulk_g2s(dk, kp, kPageRowFloats * 4, &full[st]);
        bulk_g2s(dk + kPageRowFloats, vp, kPageRowFloats * 4, &full[st]);
    };

    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) mbar_init(&full[s], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        for (int i = 0; i < kStages && i < np; ++i) issue(i);
    }

    // q slice of this lane, pre-rotated so register index i pairs with chunk c_i
    int c[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) c[i] = (((i + j) & 3) << 2) + p;
    float4 qr[HPC][4];
#pragma unroll
    for (int h = 0; h < HPC; ++h) {
        const float4* q4 = reinterpret_cast<const float4*>(a.q + ((size_t)seq * a.n_heads + h0 + h) * kHeadDim);
#pragma unroll
        for (int i = 0; i < 4; ++i) qr[h][i] = q4[c[i]];
    }
    float acc[HPC][16];
    float m[HPC], l[HPC];
#pragma unroll
    for (int h = 0; h < HPC; ++h) {
        m[h] = -INFINITY;
        l[h] = 0.f;
#pragma unroll
        for (int e = 0; e < 16; ++e) acc[h][e] = 0.f;
    }
    __syncthreads();

    const long long win_lo = S.base, win_hi = S.base + S.len;
    for (int i = 0; i < np; ++i) {
        const int st = i % kStages;
        const bool ok = mbar_wait_bounded(&full[st], (unsigned)((i / kStages) & 1));
        if (__syncthreads_or(!ok)) {
            // give up: record, drain our own copies still in flight, return
            if (tid == 0) {
                atomicExch(a.err, kErrWaitTimeout);
                const int issued = np < i + kStages ? np : i + kStages;
                for (int k = i; k < issued; ++k)
                    mbar_wait_bounded(&full[k % kStages], (unsigned)((k / kStages) & 1));
            }
            return;
        }
        const float4* Ks = reinterpret_cast<const float4*>(stages + (size_t)st * (2 * kPageRowFloats));
        const float4* Vs = Ks + kPageRowFloats / 4;
        const long long slot0 = (p0 + i) << 6;

        float s[2][HPC];
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const int row = 16 * warp + 8 * r + j;
            const long long slot = slot0 + row;
            const bool valid = slot >= win_lo && slot < win_hi;
            float4 kk[4];
#pragma unroll
            for (int ii = 0; ii < 4; ++ii) kk[ii] = Ks[row * 16 + c[ii]];
#pragma unroll
            for (int h = 0; h < HPC; ++h) {
                float d = 0.f;
#pragma unroll
                for (int ii = 0; ii < 4; ++ii) {
                    d = fmaf(qr[h][ii].x, kk[ii].x, d);
                    d = fmaf(qr[h][ii].y, kk[ii].y, d);
                    d = fmaf(qr[h][ii].z, kk[ii].z, d);
                    d = fmaf(qr[h][ii].w, kk[ii].w, d);
                }
                d += __shfl_xor_sync(0xffffffffu, d, 1);
                d += __shfl_xor_sync(0xffffffffu, d, 2);
                s[r][h] = valid ? d * a.scale_log2 : -INFINITY;
            }
        }
        float pr[2][HPC];
#pragma unroll
        for (int h = 0; h < HPC; ++h) {
            float mx = fmaxf(s[0][h], s[1][h]);
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
            if (mx > m[h]) {  // warp-uniform
                const float alpha = fast_exp2(m[h] - mx);  // m = -inf gives 0
                l[h] *= alpha;
#pragma unroll
                for (int e = 0; e < 16; ++e) acc[h][e] *= alpha;
                m[h] = mx;
            }
            const bool any = m[h] != -INFINITY;
            pr[0][h] = any ? fast_exp2(s[0][h] - m[h]) : 0.f;
            pr[1][h] = any ? fast_exp2(s[1][h] - m[h]) : 0.f;
            l[h] += pr[0][h] + pr[1][h];
        }
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const int row = 16 * warp + 8 * r + j;
            float4 vv[4];
#pragma unroll
            for (int ii = 0; ii < 4; ++ii) vv[ii] = Vs[row * 16 + c[ii]];
#pragma unroll
            for (int h = 0; h < HPC; ++h) {
                const float w = pr[r][h];
#pragma unroll
                for (int ii = 0; ii < 4; ++ii) {
                    acc[h][4 * ii + 0] = fmaf(w, vv[ii].x, acc[h][4 * ii + 0]);
                    acc[h][4 * ii + 1] = fmaf(w, vv[ii].y, acc[h][4 * ii + 1]);
                    acc[h][4 * ii + 2] = fmaf(w, vv[ii].z, acc[h][4 * ii + 2]);
                    acc[h][4 * ii + 3] = fmaf(w, vv[ii].w, acc[h][4 * ii + 3]);
                }
            }
        }
        __syncthreads();  // every warp is done with stage st
        if (tid == 0 && i + kStages < np) issue(i + kStages);
    }

    // ---- merge the 32 row-lanes x 4 warps of this CTA --------------------
#pragma unroll
    for (int h = 0; h < HPC; ++h) {
        l[h] += __shfl_xor_sync(0xffffffffu, l[h], 4);
        l[h] += __shfl_xor_sync(0xffffffffu, l[h], 8);
        l[h] += __shfl_xor_sync(0xffffffffu, l[h], 16);
    }
    float* red = stages;  // [4 warps][8 j][HPC][64]; the ring is idle now
#pragma unroll
    for (int h = 0; h < HPC; ++h) {
        float* dst = red + ((size_t)(warp * 8 + j) * HPC + h) * kHeadDim;
#pragma unroll
        for (int ii = 0; ii < 4; ++ii)
            *reinterpret_cast<float4*>(dst + 4 * c[ii]) =
                make_float4(acc[h][4 * ii], acc[h][4 * ii + 1], acc[h][4 * ii + 2], acc[h][4 * ii + 3]);
        if (lane == 0) {
            s_m[warp][h] = m[h];
            s_l[warp][h] = l[h];
        }
    }
    __syncthreads();

    const bool single = S.n_splits == 1;
    for (int o = tid; o < HPC * kHeadDim; o += kThreads) {
        const int h = o / kHeadDim, d = o % kHeadDim;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < 4; ++w) M = fmaxf(M, s_m[w][h]);
        float A = 0.f, L = 0.f;
        if (M != -INFINITY) {
#pragma unroll
            for (int w = 0; w < 4; ++w) {
                const float f = fast_exp2(s_m[w][h] - M);
                float sum = 0.f;
#pragma unroll
                for (int jj = 0; jj < 8; ++jj) sum += red[((size_t)(w * 8 + jj) * HPC + h) * kHeadDim + d];
                A = fmaf(f, sum, A);
                L = fmaf(f, s_l[w][h], L);
            }
        }
        if (single) {
            a.out[((size_t)seq * a.n_heads + h0 + h) * kHeadDim + d] = L > 0.f ? A / L : 0.f;
        } else {
            const size_t pi = ((size_t)gsplit * NY + y) * HPC + h;
            a.part_acc[pi * kHeadDim + d] = A;
            if (d == 0) {
                a.part_ml[pi * 2 + 0] = M;
                a.part_ml[pi * 2 + 1] = L;
            }
        }
    }
    if (single) return;

    // ---- last CTA of this (sequence, kv head) merges the splits ----------
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        unsigned* ctr = a.counters + (size_t)seq * NY + y;
        const unsigned prev = atomicAdd(ctr, 1u);
        s_last = (prev == (unsigned)(S.n_splits - 1));
        if (s_last) *ctr = 0u;  // ready for the next launch
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    for (int o = tid; o < HPC * kHeadDim; o += kThreads) {
        const int h = o / kHeadDim, d = o % kHeadDim;
        float M = -INFINITY;
        for (int k = 0; k < S.n_splits; ++k) {
            const size_t pi = ((size_t)(S.split0 + k) * NY + y) * HPC + h;
            M = fmaxf(M, __ldcg(a.part_ml + pi * 2));
        }
        float A = 0.f, L = 0.f;
        if (M != -INFINITY) {
            for (int k = 0; k < S.n_splits; ++k) {
                const size_t pi = ((size_t)(S.split0 + k) * NY + y) * HPC + h;
                const float mk = __ldcg(a.part_ml + pi * 2);
                const float f = fast_exp2(mk - M);
                A = fmaf(f, __ldcg(a.part_acc + pi * kHeadDim + d), A);
                L = fmaf(f, __ldcg(a.part_ml + pi * 2 + 1), L);
            }
        }
        a.out[((size_t)seq * a.n_heads + h0 + h) * kHeadDim + d] = L > 0.f ? A / L : 0.f;
    }
}

template <int HPC>
cudaError_t launch_hpc(const DecodeArgs& a, cudaStream_t s) {
    static bool attr_set = false;  // per process; the attribute is per device function
    const int smem = (int)decode_smem_bytes();
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(decode_kernel<HPC>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        attr_set = true;
    }
    dim3 grid((unsigned)a.total_splits, (unsigned)(a.n_kv * a.n_sub));
    decode_kernel<HPC><<<grid, kThreads, smem, s>>>(a);
    return cudaGetLastError();
}

}  // namespace

size_t decode_smem_bytes() { return (size_t)kStages * kStageBytes + kStages * sizeof(uint64_t); }

cudaError_t launch_decode(const DecodeArgs& a, cudaStream_t s) {
    if (a.total_splits <= 0) return cudaSuccess;
    switch (a.hpc) {
        case 1: return launch_hpc<1>(a, s);
        case 2: return launch_hpc<2>(a, s);
        case 3: return launch_hpc<3>(a, s);
        case 4: return launch_hpc<4>(a, s);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace bebelm
