// Q4_K x Q8 matmul on the 5th-generation tensor cores (many tokens).
//
// The same arithmetic as qmatmul_tiled_kernel (quant.cu), which restates the reference's
// dot_q4k_block_q8 (src/kernels/matmul.rs:220-244): per 256-weight block of a row and a token,
//     sd = Σ_j sc_j · <nibbles_j, q_j>,   sm = Σ_j m_j · Σ_{k in j} q_k,
//     value = sx * (d * sd - dmin * sm)   (f32, no contraction), blocks added in order from -0.
// sd and sm are exact integers, so any exact way of forming them gives the reference's bits.
// Here the tensor cores form them (`tcgen05.mma kind::i8`, s8 x s8 -> s32, K = 32 per MMA):
//     sd = Σ_k (nib_k · (sc_j & 7)) q_k  +  8 · Σ_k (nib_k · (sc_j >> 3)) q_k
//     sm = Σ_k m_j q_k
// Every A operand stays within s8 (15·7 = 105, m_j <= 63), so a block is 3 x 8 MMAs into 3 s32
// accumulators (lo, hi, min) of 128 rows x 64 tokens, and the epilogue per (row, token) is one
// shift-add and the f32 expression above.
//
// One CTA per (128 rows, 64 tokens), 16 warps, one CTA per SM (shared memory). Per block b:
//   * cp.async, one block ahead, into a 3-stage ring: the 128 rows' raw 144-byte blocks, the
//     64 tokens' Q8 activations written straight into the 128-byte-swizzled K-major layout the
//     MMA reads as B, and their scales;
//   * wait for block b-1's MMAs (they read the single A buffer), then unpack block b's nibbles,
//     scales and mins into the three A tiles (128-byte-swizzled, K-major);
//   * one thread issues the 24 MMAs into TMEM buffer b & 1 and commits them to an mbarrier;
//   * meanwhile all threads run block b-1's epilogue from TMEM buffer (b-1) & 1: thread
//     (row, quarter) adds 16 tokens' block values to its running sums.
// Every mbarrier wait is bounded (one thread polls, the CTA barrier passes its result on): on
// timeout the CTA records kErrWaitTimeout, waits for its own copies, frees its TMEM and returns
// without storing.
#include "internal.h"

namespace bebelm {
namespace {

constexpr int kQK = 256;
constexpr int kM = 128, kN = 64, kThreads = 512, kStages = 3;
constexpr int kAtomA = kM * 128;  // one 128-byte-wide swizzle atom of A (K 0..127 or 128..255): 16 KB
constexpr int kAtomB = kN * 128;  // of B: 8 KB
constexpr int kTileA = 2 * kAtomA, kTileB = 2 * kAtomB;
constexpr int kRawRow = 144;
constexpr int kOffA = 0;                                   // A tiles: lo, hi, min
constexpr int kOffB = kOffA + 3 * kTileA;                  // kStages x B tile
constexpr int kOffRaw = kOffB + kStages * kTileB;          // kStages x 128 rows x 144 B
constexpr int kOffSx = kOffRaw + kStages * kM * kRawRow;   // kStages x 64 floats
constexpr int kOffBar = kOffSx + kStages * kN * 4;
constexpr int kSmemBytes = kOffBar + 64 + 1024;            // + alignment slack
constexpr uint32_t kTmemCols = 512;                        // 2 buffers x 3 accumulators x 64 columns
constexpr long long kWaitLimit = 1ll << 22;

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0) : "memory");
}
__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src, bool valid) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src), "r"(valid ? 4 : 0) : "memory");
}

// byte offset of (row, k) in a K-major tile of two 128-byte-swizzled atoms (K 0..127, 128..255):
// inside an atom, 8-row groups of 1024 bytes, the 16-byte chunk index XORed with the row in its group
template <int kAtom>
__device__ __forceinline__ uint32_t swz(int row, int k) {
    const uint32_t o = (uint32_t)(row * 128 + (k & 127));
    return (uint32_t)(k >> 7) * kAtom + (o ^ (((o >> 7) & 7u) << 4));
}

__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {  // 128B swizzle, K-major, SBO 1024, version 1
    return (uint64_t)((addr & 0x3FFFF) >> 4) | ((uint64_t)(16 >> 4) << 16) | ((uint64_t)(1024 >> 4) << 32) |
           (1ull << 46) | (2ull << 61);
}
// kind::i8: D s32 (2 at bit 4), A and B signed 8-bit (1 at bits 7 and 10), both K-major, N, M
constexpr uint32_t kIdesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kN >> 3) << 17) | ((uint32_t)(kM >> 4) << 24);

__device__ __forceinline__ bool mbar_wait(uint32_t bar, unsigned parity) {
    for (long long it = 0; it < kWaitLimit; ++it) {
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

// 32 lanes x 16 consecutive 32-bit TMEM columns (no wait; tmem_wait() before use)
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, int* v) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
          "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tc_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ float f16f(uint32_t h) {
    __half_raw r;
    r.x = (unsigned short)h;
    return __half2float(__half(r));
}

__global__ void __launch_bounds__(kThreads, 1) q4k_tc_kernel(const uint8_t* w, size_t row_bytes, size_t n_in,
                                                             size_t n_out, size_t n_tokens, const int8_t* q8,
                                                             const float* q8_scales, float* y, int* err) {
    extern __shared__ unsigned char smem_raw[];
    unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sb = smem_u32(sm);
    __shared__ uint32_t s_tmem;
    const int tid = threadIdx.x, warp = tid >> 5;
    const size_t r0 = (size_t)blockIdx.x * kM, t0 = (size_t)blockIdx.y * kN;
    const size_t nb = n_in / kQK;
    const uint32_t bar = sb + kOffBar;

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    if (tid == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    tc_before();
    __syncthreads();
    tc_after();
    const uint32_t tmem = s_tmem;

    // one block's operands into ring stage st, asynchronously (one commit group). A thread's
    // copy tasks are the same for every block: 16-byte pieces of the raw rows (9 per row) and
    // of the activations (16 per token), their sources advancing by one block each time.
    constexpr int kRawTasks = (kM * 9 + kThreads - 1) / kThreads, kBTasks = kN * 16 / kThreads;
    const uint8_t* raw_src[kRawTasks];
    uint32_t raw_dst[kRawTasks];
    bool raw_ok[kRawTasks];
#pragma unroll
    for (int i = 0; i < kRawTasks; ++i) {
        const int task = tid + i * kThreads, r = task / 9, seg = task - 9 * r;
        raw_ok[i] = task < kM * 9 && r0 + r < n_out;
        raw_src[i] = raw_ok[i] ? w + (r0 + r) * row_bytes + seg * 16 : w;
        raw_dst[i] = task < kM * 9 ? (uint32_t)(kOffRaw + r * kRawRow + seg * 16) : 0xffffffffu;
    }
    const int8_t* b_src[kBTasks];
    uint32_t b_dst[kBTasks];
    bool b_ok[kBTasks];
#pragma unroll
    for (int i = 0; i < kBTasks; ++i) {
        const int task = tid + i * kThreads, t = task >> 4, k = (task & 15) * 16;
        b_ok[i] = t0 + t < n_tokens;
        b_src[i] = b_ok[i] ? q8 + (t0 + t) * n_in + k : q8;
        b_dst[i] = (uint32_t)kOffB + swz<kAtomB>(t, k);
    }
    const bool sx_ok = tid < kN && t0 + tid < n_tokens;
    const float* sx_src = sx_ok ? q8_scales + (t0 + tid) * nb : q8_scales;
    auto stage = [&](size_t bb, int st) {
#pragma unroll
        for (int i = 0; i < kRawTasks; ++i)
            if (raw_dst[i] != 0xffffffffu)
                cp_async16(sb + raw_dst[i] + st * kM * kRawRow, raw_ok[i] ? raw_src[i] + bb * 144 : w, raw_ok[i]);
#pragma unroll
        for (int i = 0; i < kBTasks; ++i)
            cp_async16(sb + b_dst[i] + st * kTileB, b_ok[i] ? b_src[i] + bb * kQK : q8, b_ok[i]);
        if (tid < kN) cp_async4(sb + kOffSx + st * kN * 4 + tid * 4, sx_ok ? sx_src + bb : q8_scales, sx_ok);
        asm volatile("cp.async.commit_group;" ::: "memory");
    };

    // unpack and epilogue roles: thread (row, quarter)
    const int row = tid & (kM - 1), quarter = tid >> 7;
    const uint32_t t_lane = tmem + ((uint32_t)(32 * (warp & 3)) << 16);
    float acc[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[i] = -0.0f;

    stage(0, 0);
    bool ok = true;
    for (size_t b = 0; b <= nb; ++b) {
        __syncthreads();  // block b-2's epilogue is done with its TMEM buffer and ring stage
        if (b < nb) {
            if (b + 1 < nb)
                stage(b + 1, (int)((b + 1) % kStages));
            else
                asm volatile("cp.async.commit_group;" ::: "memory");
            asm volatile("cp.async.wait_group 1;" ::: "memory");  // block b's operands have landed
        }
        if (b >= 1) {  // block b-1's MMAs: A is free, its accumulators are complete
            // one thread polls while the others sleep in the CTA barrier; then every thread
            // acquires the completed phase itself (one try_wait that succeeds at once), which is
            // what orders its TMEM loads after the MMAs
            const unsigned par = (unsigned)((b - 1) & 1);
            const bool mine = tid == 0 ? mbar_wait(bar, par) : true;
            if (__syncthreads_or(!mine)) {
                ok = false;
                break;
            }
            if (tid != 0) mbar_wait(bar, par);
            tc_after();
        }
        if (b < nb) {
            const int st = (int)(b % kStages);
            // unpack chunk `quarter` (64 weights: sub-blocks 2q (low nibbles), 2q+1 (high)) of `row`
            const unsigned char* raw = sm + kOffRaw + st * kM * kRawRow + row * kRawRow;
            const uint4 sc4 = *reinterpret_cast<const uint4*>(raw);  // d, dmin, scales[0..11]
            const uint32_t s0 = sc4.y, s1 = sc4.z, s2 = sc4.w;       // scale bytes 0-3, 4-7, 8-11
            uint32_t sc[2], mn[2];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int j = 2 * quarter + h;
                // 6-bit scale and min of sub-block j (ggml's get_scale_min_k4)
                if (j < 4) {
                    sc[h] = (s0 >> (8 * j)) & 63;
                    mn[h] = (s1 >> (8 * j)) & 63;
                } else {
                    const uint32_t b8 = (s2 >> (8 * (j - 4))) & 0xff;
                    sc[h] = (b8 & 0x0f) | (((s0 >> (8 * (j - 4) + 6)) & 3) << 4);
                    mn[h] = (b8 >> 4) | (((s1 >> (8 * (j - 4) + 6)) & 3) << 4);
                }
            }
#pragma unroll
            for (int p = 0; p < 32; p += 16) {
                const uint4 q = *reinterpret_cast<const uint4*>(raw + 16 + quarter * 32 + p);
                const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    uint32_t lo[4], hi[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const uint32_t nib = h ? (qw[e] >> 4) & 0x0f0f0f0fu : qw[e] & 0x0f0f0f0fu;
                        lo[e] = nib * (sc[h] & 7);  // bytewise: 15 * 7 < 256, no carries
                        hi[e] = nib * (sc[h] >> 3);
                    }
                    const uint32_t m4 = mn[h] * 0x01010101u;
                    const int k = (2 * quarter + h) * 32 + p;
                    const uint32_t off = swz<kAtomA>(row, k);
                    *reinterpret_cast<uint4*>(sm + kOffA + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
                    *reinterpret_cast<uint4*>(sm + kOffA + kTileA + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                    *reinterpret_cast<uint4*>(sm + kOffA + 2 * kTileA + off) = make_uint4(m4, m4, m4, m4);
                }
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // A and B (cp.async) -> tensor core
            tc_before();
            __syncthreads();
            if (tid == 0) {
                tc_after();
                const uint32_t bB = sb + kOffB + st * kTileB, dbuf = tmem + (uint32_t)(b & 1) * 256;
#pragma unroll
                for (int a = 0; a < 3; ++a) {
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk) {  // K step: atom kk / 4, 32 bytes at (kk % 4) * 32
                        const uint32_t koff = (uint32_t)(kk & 3) * 32;
                        const uint64_t ad = smem_desc(sb + kOffA + a * kTileA + (kk >> 2) * kAtomA + koff);
                        const uint64_t bd = smem_desc(bB + (kk >> 2) * kAtomB + koff);
                        asm volatile(
                            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                            "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(dbuf + a * kN),
                            "l"(ad), "l"(bd), "r"(kIdesc), "r"(kk)
                            : "memory");
                    }
                }
                asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                             : "memory");
            }
        }
        if (b >= 1) {  // epilogue of block b-1: (row, tokens 16 quarter .. +15)
            const size_t bp = b - 1;
            const int st = (int)(bp % kStages);
            const uint32_t* head = reinterpret_cast<const uint32_t*>(sm + kOffRaw + st * kM * kRawRow + row * kRawRow);
            const float d = f16f(head[0] & 0xffffu), dmin = f16f(head[0] >> 16);
            const uint32_t tb = t_lane + (uint32_t)(bp & 1) * 256 + 16 * quarter;
            int lo[16], hi[16], mv[16];
            tmem_ld16(tb, lo);
            tmem_ld16(tb + kN, hi);
            tmem_ld16(tb + 2 * kN, mv);
            tmem_wait();
            const float* sx = reinterpret_cast<const float*>(sm + kOffSx + st * kN * 4) + 16 * quarter;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const int sd = lo[i] + 8 * hi[i];
                const float v = __fmul_rn(sx[i], __fsub_rn(__fmul_rn(d, __int2float_rn(sd)),
                                                           __fmul_rn(dmin, __int2float_rn(mv[i]))));
                acc[i] = __fadd_rn(acc[i], v);
            }
            tc_before();
        }
    }
    if (ok) {
        const size_t r = r0 + row;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const size_t t = t0 + 16 * quarter + i;
            if (r < n_out && t < n_tokens) y[t * n_out + r] = acc[i];
        }
    } else if (tid == 0) {
        *reinterpret_cast<volatile int*>(err) = kErrWaitTimeout;
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();
    if (warp == 0) {
        tc_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
    }
}

}  // namespace

cudaError_t launch_q4k_tc(const uint8_t* w, size_t n_in, size_t n_out, size_t n_tokens, const int8_t* q8,
                          const float* q8_scales, float* y, int* err, cudaStream_t s) {
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(q4k_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) attr_set[dev] = true;
    }
    const dim3 grid((unsigned)((n_out + kM - 1) / kM), (unsigned)((n_tokens + kN - 1) / kN));
    q4k_tc_kernel<<<grid, kThreads, kSmemBytes, s>>>(w, n_in / kQK * 144, n_in, n_out, n_tokens, q8, q8_scales, y, err);
    return cudaGetLastError();
}

}  // namespace bebelm
