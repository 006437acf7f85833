// Kernel 2: causal prefill attention on the 5th-generation tensor cores.
//
// Computes, for a chunk of t queries appended after len_before cached positions
// (the reference's `attn_batch`, src/model.rs:232-254, where token i runs
// `attention_decode` over the len_before + i + 1 keys present once its own k/v
// is appended), out[i, h] = Σ_{j <= len_before+i} softmax_j(q_i·k_j * scale) v_j
// with bf16 operands and fp32 accumulation, as a flash-attention loop.
//
// One CTA per (128-query tile, query head); 128 threads = 4 warps, warp w owns
// TMEM lanes / query rows 32w..32w+31.
//   * TMA (cp.async.bulk.tensor, 128-byte swizzle) brings the Q tile once and
//     K/V tiles of 128 keys into a 2-deep ring.
//   * Thread 0 issues S = Q Kᵀ as 4 tcgen05.mma (M=128, N=128, K=16) into
//     TMEM columns [0,128) and commits to an mbarrier.
//   * Every thread loads its S row from TMEM (tcgen05.ld 32x32b), applies the
//     causal mask and the online softmax in fp32 (exp2 with log2e folded into
//     the scale), and writes P in bf16 to shared memory in the 128-byte-swizzled
//     K-major layout the MMA reads.
//   * Thread 0 issues O_tile = P V as 8 tcgen05.mma (N=64, K=16, V read
//     MN-major) into TMEM columns [128,192); each thread folds its row into the
//     fp32 output held in registers with the running rescale.
// Tiles entirely above the diagonal are never visited. Every mbarrier wait is
// bounded: on timeout the CTA records kErrWaitTimeout, waits (bounded) for its
// own copies and MMAs, frees its TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "internal.h"

namespace bebelm {
namespace {

constexpr int kThreads = 128;
constexpr int kTileQ = 128, kTileK = 128;
constexpr int kTileBytes = kTileQ * kHeadDim * 2;  // 16 KB: 128 rows x 128 B
constexpr int kTmemCols = 256;                     // S: [0,128), O tile: [128,192)
constexpr long long kWaitLimit = 1ll << 22;

// shared memory map (offsets from a 1024-byte aligned base)
constexpr int kOffQ = 0;
constexpr int kOffK = kOffQ + kTileBytes;           // 2 buffers
constexpr int kOffV = kOffK + 2 * kTileBytes;       // 2 buffers
constexpr int kOffP = kOffV + 2 * kTileBytes;       // 2 blocks of 64 keys
constexpr int kOffBar = kOffP + 2 * kTileBytes;
constexpr int kSmemBytes = kOffBar + 64 + 1024;     // barriers + alignment slack

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint32_t bar, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, unsigned parity) {
    for (long long it = 0; it < kWaitLimit; ++it) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(bar), "r"(parity)
            : "memory");
        if (ok) return true;
    }
    return false;
}
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2,
                                            uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(dst),
        "l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(bar)
        : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor: 128-byte swizzle, version 1 (sm_100).
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((addr & 0x3FFFF) >> 4) | ((uint64_t)(lbo >> 4) << 16) | ((uint64_t)(sbo >> 4) << 32) |
           (1ull << 46) | (2ull << 61);
}

// Instruction descriptor, kind::f16: bf16 x bf16 -> f32, M = 128.
__host__ __device__ constexpr uint32_t instr_desc(int n, bool b_mn_major) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((b_mn_major ? 1u : 0u) << 16) | ((uint32_t)(n >> 3) << 17) |
           ((uint32_t)(128 >> 4) << 24);
}

__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

// 32 lanes x 32 consecutive columns of 32-bit TMEM cells into 32 registers per thread.
// The wait sits in the same asm statement, so no use of the registers can be
// scheduled before the load has completed.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

__global__ void __launch_bounds__(kThreads, 1)
    prefill_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                   const __grid_constant__ CUtensorMap tm_v, PrefillArgs a) {
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sbase = smem_u32(smem);
    const uint32_t bar_q = sbase + kOffBar, bar_kv0 = bar_q + 8, bar_s = bar_q + 24, bar_o = bar_q + 32;
    __shared__ uint32_t s_tmem;
    __shared__ int s_fail;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n_qt = (a.t + kTileQ - 1) / kTileQ;
    const int qt = n_qt - 1 - (int)blockIdx.x;  // longest rows first
    const int h = blockIdx.y, kvh = h / (a.n_heads / a.n_kv);
    const int q0 = qt * kTileQ;
    const int q_last = min(q0 + kTileQ, a.t) - 1;
    const int n_kt = (a.len_before + q_last) / kTileK + 1;

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    if (tid == 0) {
        s_fail = 0;
        for (int i = 0; i < 5; ++i) mbar_init(bar_q + 8 * i, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_expect_tx(bar_q, kTileBytes);
        tma_load_3d(sbase + kOffQ, &tm_q, 0, h, q0, bar_q);
        for (int i = 0; i < 2 && i < n_kt; ++i) {
            mbar_expect_tx(bar_kv0 + 8 * i, 2 * kTileBytes);
            tma_load_3d(sbase + kOffK + i * kTileBytes, &tm_k, 0, kvh, i * kTileK, bar_kv0 + 8 * i);
            tma_load_3d(sbase + kOffV + i * kTileBytes, &tm_v, 0, kvh, i * kTileK, bar_kv0 + 8 * i);
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    const uint32_t t_row = tmem + ((uint32_t)(32 * warp) << 16);  // this warp's TMEM lanes

    const int row = 32 * warp + lane;
    const int qi = q0 + row;
    const long long key_lim = (long long)a.len_before + qi;  // last key this row may see
    float o[kHeadDim];
#pragma unroll
    for (int d = 0; d < kHeadDim; ++d) o[d] = 0.f;
    float m = -INFINITY, l = 0.f;
    constexpr uint32_t kIdescS = instr_desc(kTileK, false), kIdescO = instr_desc(kHeadDim, true);
    bool failed = false;
    int kt = 0;
    for (; kt < n_kt; ++kt) {
        const int b = kt & 1;
        // ---- S = Q K^T ------------------------------------------------------
        if (tid == 0) {
            bool ok = (kt > 0 || mbar_wait_bounded(bar_q, 0)) && mbar_wait_bounded(bar_kv0 + 8 * b, (kt >> 1) & 1);
            if (ok) {
                tc_fence_after();
                const uint32_t qa = sbase + kOffQ, ka = sbase + kOffK + b * kTileBytes;
#pragma unroll
                for (int k = 0; k < kHeadDim / 16; ++k)
                    mma_bf16(tmem, smem_desc(qa + 32 * k, 16, 1024), smem_desc(ka + 32 * k, 16, 1024), kIdescS, k > 0);
                mma_commit(bar_s);
            } else {
                s_fail = 1;
            }
        }
        const bool ok_s = mbar_wait_bounded(bar_s, kt & 1);
        if (__syncthreads_or(!ok_s || s_fail)) {
            failed = true;
            break;
        }
        tc_fence_after();
        // ---- online softmax on this thread's row -----------------------------
        float s[kTileK];
#pragma unroll
        for (int c = 0; c < kTileK; c += 32) tmem_ld32(t_row + c, s + c);
        const long long k0 = (long long)kt * kTileK;
        float mx = m;
#pragma unroll
        for (int c = 0; c < kTileK; ++c) {
            s[c] = (k0 + c <= key_lim) ? s[c] * a.scale_log2 : -INFINITY;
            mx = fmaxf(mx, s[c]);
        }
        const float alpha = exp2f(m - mx);  // m = -inf gives 0
        m = mx;
        float psum = 0.f;
        unsigned char* pbase = smem + kOffP;
#pragma unroll
        for (int c = 0; c < kTileK; c += 8) {
            float p[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                p[e] = exp2f(s[c + e] - mx);
                psum += p[e];
            }
            uint4 w = make_uint4(pack_bf16(p[0], p[1]), pack_bf16(p[2], p[3]), pack_bf16(p[4], p[5]),
                                 pack_bf16(p[6], p[7]));
            const int blk = c >> 6, chunk = (c & 63) >> 3;
            *reinterpret_cast<uint4*>(pbase + blk * kTileBytes + row * 128 + ((chunk ^ (row & 7)) << 4)) = w;
        }
        l = l * alpha + psum;
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        tc_fence_before();
        __syncthreads();
        // ---- O_tile = P V ----------------------------------------------------
        if (tid == 0) {
            tc_fence_after();
            const uint32_t pa = sbase + kOffP, va = sbase + kOffV + b * kTileBytes;
#pragma unroll
            for (int k = 0; k < kTileK / 16; ++k)
                mma_bf16(tmem + 128, smem_desc(pa + (k >> 2) * kTileBytes + 32 * (k & 3), 16, 1024),
                         smem_desc(va + 2048 * k, kTileBytes, 1024), kIdescO, k > 0);
            mma_commit(bar_o);
        }
        const bool ok_o = mbar_wait_bounded(bar_o, kt & 1);
        if (__syncthreads_or(!ok_o)) {
            failed = true;
            break;
        }
        tc_fence_after();
        float pv[kHeadDim];
        tmem_ld32(t_row + 128, pv);
        tmem_ld32(t_row + 160, pv + 32);
#pragma unroll
        for (int d = 0; d < kHeadDim; ++d) o[d] = fmaf(o[d], alpha, pv[d]);
        tc_fence_before();
        __syncthreads();  // S, P and this K/V buffer are free again
        if (tid == 0 && kt + 2 < n_kt) {
            mbar_expect_tx(bar_kv0 + 8 * b, 2 * kTileBytes);
            tma_load_3d(sbase + kOffK + b * kTileBytes, &tm_k, 0, kvh, (kt + 2) * kTileK, bar_kv0 + 8 * b);
            tma_load_3d(sbase + kOffV + b * kTileBytes, &tm_v, 0, kvh, (kt + 2) * kTileK, bar_kv0 + 8 * b);
        }
    }

    if (failed) {
        if (tid == 0) {
            atomicExch(a.err, kErrWaitTimeout);
            // let whatever this CTA started land before its memory goes away
            mbar_wait_bounded(bar_q, 0);
            for (int k = kt; k < kt + 2 && k < n_kt; ++k) mbar_wait_bounded(bar_kv0 + 8 * (k & 1), (k >> 1) & 1);
            mbar_wait_bounded(bar_s, kt & 1);
            mbar_wait_bounded(bar_o, kt & 1);
        }
    } else if (qi < a.t) {
        const float inv = l > 0.f ? 1.f / l : 0.f;
        float4* dst = reinterpret_cast<float4*>(a.out + ((size_t)qi * a.n_heads + h) * kHeadDim);
#pragma unroll
        for (int d = 0; d < kHeadDim; d += 4)
            dst[d / 4] = make_float4(o[d] * inv, o[d + 1] * inv, o[d + 2] * inv, o[d + 3] * inv);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
    }
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

// [rows][heads][64] bf16 viewed as a 3-D tensor (d, head, row); box = one head x 128 rows.
bool make_map(CUtensorMap* m, const void* base, int heads, long long rows) {
    auto enc = tensor_map_encoder();
    if (!enc) return false;
    cuuint64_t dims[3] = {(cuuint64_t)kHeadDim, (cuuint64_t)heads, (cuuint64_t)rows};
    cuuint64_t strides[2] = {(cuuint64_t)kHeadDim * 2, (cuuint64_t)heads * kHeadDim * 2};
    cuuint32_t box[3] = {(cuuint32_t)kHeadDim, 1, 128};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

}  // namespace

cudaError_t launch_prefill(const PrefillArgs& a, cudaStream_t s) {
    if (a.t <= 0) return cudaSuccess;
    CUtensorMap mq, mk, mv;
    const long long s_total = (long long)a.len_before + a.t;
    if (!make_map(&mq, a.q, a.n_heads, a.t) || !make_map(&mk, a.k, a.n_kv, s_total) ||
        !make_map(&mv, a.v, a.n_kv, s_total))
        return cudaErrorInvalidValue;
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) attr_set[dev] = true;
    }
    dim3 grid((unsigned)((a.t + kTileQ - 1) / kTileQ), (unsigned)a.n_heads);
    prefill_kernel<<<grid, kThreads, kSmemBytes, s>>>(mq, mk, mv, a);
    return cudaGetLastError();
}

}  // namespace bebelm
