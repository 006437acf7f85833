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
constexpr int kPrefetch = 2;                          // pages prefetched into L2 beyond the ring

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

__device__ __forceinline__ void bulk_prefetch_l2(const void* src, unsigned bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

template <int HPC>
__global__ void __launch_bounds__(kThreads, 2) decode_kernel(DecodeArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    float* stages = reinterpret_cast<float*>(smem);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
    __shared__ float s_m[4][HPC], s_l[4][HPC];
    __shared__ int s_release[kStages];
    __shared__ int s_failed;
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

    auto page_src = [&](int i) -> const float* {
        const long long lp = p0 + i;
        const int phys = S.table[(int)(lp % S.cap)];
        return a.pv.base + (size_t)phys * a.pv.page_floats + a.pv.layer_off + (size_t)kvh * kPageRowFloats;
    };
    auto issue = [&](int i) {
        const int st = i % kStages;
        const float* kp = page_src(i);
        float* dk = stages + (size_t)st * (2 * kPageRowFloats);
        mbar_expect_tx(&full[st], kStageBytes);
        bulk_g2s(dk, kp, kPageRowFloats * 4, &full[st]);
        bulk_g2s(dk + kPageRowFloats, kp + a.pv.block_floats, kPageRowFloats * 4, &full[st]);
    };
    auto prefetch = [&](int i) {
        const float* kp = page_src(i);
        bulk_prefetch_l2(kp, kPageRowFloats * 4);
        bulk_prefetch_l2(kp + a.pv.block_floats, kPageRowFloats * 4);
    };

    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            s_release[s] = 0;
        }
        s_failed = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        for (int i = 0; i < kStages && i < np; ++i) issue(i);
        for (int i = kStages; i < kStages + kPrefetch && i < np; ++i) prefetch(i);
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
    int consumed = 0;  // pages this warp finished (the rest are still owed to the ring)
    for (int i = 0; i < np; ++i) {
        const int st = i % kStages;
        const bool ok = __all_sync(0xffffffffu, mbar_wait_bounded(&full[st], (unsigned)((i / kStages) & 1)));
        if (!ok) {
            if (lane == 0) {
                atomicExch(a.err, kErrWaitTimeout);
                atomicExch(&s_failed, 1);
            }
            break;
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
        float4 vv[2][4];
#pragma unroll
        for (int r = 0; r < 2; ++r)
#pragma unroll
            for (int ii = 0; ii < 4; ++ii) vv[r][ii] = Vs[(16 * warp + 8 * r + j) * 16 + c[ii]];
        // V is in registers: this warp is done with the stage
        __syncwarp();
        if (lane == 0) {
            if (atomicAdd(&s_release[st], 1) == 3) {  // last of the 4 warps refills the stage
                s_release[st] = 0;
                if (i + kStages < np) {
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    issue(i + kStages);
                    if (i + kStages + kPrefetch < np) prefetch(i + kStages + kPrefetch);
                }
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
#pragma unroll
            for (int h = 0; h < HPC; ++h) {
                const float w = pr[r][h];
#pragma unroll
                for (int ii = 0; ii < 4; ++ii) {
                    acc[h][4 * ii + 0] = fmaf(w, vv[r][ii].x, acc[h][4 * ii + 0]);
                    acc[h][4 * ii + 1] = fmaf(w, vv[r][ii].y, acc[h][4 * ii + 1]);
                    acc[h][4 * ii + 2] = fmaf(w, vv[r][ii].z, acc[h][4 * ii + 2]);
                    acc[h][4 * ii + 3] = fmaf(w, vv[r][ii].w, acc[h][4 * ii + 3]);
                }
            }
        }
        consumed = i + 1;
    }
    (void)consumed;
    __syncthreads();
    if (s_failed) {
        // a wait gave up: let our own copies still in flight land (bounded), then leave
        if (tid == 0) {
            for (int k = 0; k < kStages && k < np; ++k) {
                // the newest issue into stage k is the largest page index < np with index % kStages == k
                const int last = ((np - 1 - k) / kStages) * kStages + k;
                mbar_wait_bounded(&full[k], (unsigned)((last / kStages) & 1));
            }
        }
        return;
    }

    // ---- merge the 8 row-lanes x 4 warps of this CTA ----------------------
#pragma unroll
    for (int h = 0; h < HPC; ++h) {
        l[h] += __shfl_xor_sync(0xffffffffu, l[h], 4);
        l[h] += __shfl_xor_sync(0xffffffffu, l[h], 8);
        l[h] += __shfl_xor_sync(0xffffffffu, l[h], 16);
    }
    float* red = stages;  // [4 warps][8 j][HPC][64]; every copy has landed and been read
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
    const int ns = S.n_splits;
    // split maxima and sums into shared memory (one load per thread, all in flight at once)
    float* sm_m = red;                  // [ns][HPC]
    float* sm_l = red + ns * HPC;       // [ns][HPC]
    for (int x = tid; x < ns * HPC; x += kThreads) {
        const size_t pi = ((size_t)(S.split0 + x / HPC) * NY + y) * HPC + (x % HPC);
        sm_m[x] = __ldcg(a.part_ml + pi * 2);
        sm_l[x] = __ldcg(a.part_ml + pi * 2 + 1);
    }
    __syncthreads();
    __shared__ float s_L[HPC];
    if (tid < HPC) {
        float M = -INFINITY;
        for (int k = 0; k < ns; ++k) M = fmaxf(M, sm_m[k * HPC + tid]);
        float L = 0.f;
        for (int k = 0; k < ns; ++k) {
            const float f = M == -INFINITY ? 0.f : fast_exp2(sm_m[k * HPC + tid] - M);
            sm_m[k * HPC + tid] = f;  // now the rescale factor of split k
            L = fmaf(f, sm_l[k * HPC + tid], L);
        }
        s_L[tid] = L;
    }
    __syncthreads();
    for (int o = tid; o < HPC * kHeadDim; o += kThreads) {
        const int h = o / kHeadDim, d = o % kHeadDim;
        float A0 = 0.f, A1 = 0.f, A2 = 0.f, A3 = 0.f;
        const float* src = a.part_acc + ((size_t)S.split0 * NY + y) * HPC * kHeadDim + (size_t)h * kHeadDim + d;
        const size_t stride = (size_t)NY * HPC * kHeadDim;
        int k = 0;
        for (; k + 4 <= ns; k += 4) {
            const float x0 = __ldcg(src + (size_t)(k + 0) * stride), x1 = __ldcg(src + (size_t)(k + 1) * stride);
            const float x2 = __ldcg(src + (size_t)(k + 2) * stride), x3 = __ldcg(src + (size_t)(k + 3) * stride);
            A0 = fmaf(sm_m[(k + 0) * HPC + h], x0, A0);
            A1 = fmaf(sm_m[(k + 1) * HPC + h], x1, A1);
            A2 = fmaf(sm_m[(k + 2) * HPC + h], x2, A2);
            A3 = fmaf(sm_m[(k + 3) * HPC + h], x3, A3);
        }
        for (; k < ns; ++k) A0 = fmaf(sm_m[k * HPC + h], __ldcg(src + (size_t)k * stride), A0);
        const float A = (A0 + A1) + (A2 + A3);
        const float L = s_L[h];
        a.out[((size_t)seq * a.n_heads + h0 + h) * kHeadDim + d] = L > 0.f ? A / L : 0.f;
    }
}

template <int HPC>
cudaError_t launch_hpc(const DecodeArgs& a, cudaStream_t s) {
    static bool attr_set[64] = {};  // the attribute is per device
    const int smem = (int)decode_smem_bytes();
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(decode_kernel<HPC>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) attr_set[dev] = true;
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
