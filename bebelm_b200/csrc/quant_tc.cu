// K-quant (Q4_K, Q6_K) x Q8 matmul on the 5th-generation tensor cores (many tokens).
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
// accumulators (lo, hi, min) of 128 rows x 128 tokens (384 TMEM columns), and the epilogue per
// (row, token) is one shift-add and the f32 expression above.
//
// One CTA per (128 rows, 128 tokens), one CTA per SM (shared memory), warp-specialised:
//   * control warp (warp 16, one lane): TMA loads of block b+2 (the 128 rows' raw 144-byte
//     blocks, and the 128 tokens' Q8 activations in the 128-byte-swizzled K-major layout the
//     MMA reads as B) into a 2-slot ring as soon as block b's MMAs have finished with its slot;
//     and the 24 MMAs of each block once the workers have unpacked it.
//   * 16 worker warps, thread (row, quarter of the tokens): for block b, wait for block b-1's
//     MMAs and block b's loads; read block b-1's accumulators from TMEM and add the block
//     values of 32 tokens to the row's running sums; unpack block b's nibbles, scales and mins
//     into the three A tiles (128-byte-swizzled, K-major); hand A to the control warp.
// Token scales are read by the workers one block ahead into registers.
// Every wait is bounded (one thread polls and the others then acquire the completed phase once):
// on timeout the CTA records kErrWaitTimeout, waits (bounded) for its loads and MMAs in flight,
// frees its TMEM and returns without storing.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "internal.h"

namespace bebelm {
namespace {

constexpr int kQK = 256;
constexpr int kM = 128, kN = 128, kWorkers = 512, kThreads = kWorkers + 32;
constexpr int kAtomA = kM * 128;  // one 128-byte-wide swizzle atom of A (K 0..127 or 128..255): 16 KB
constexpr int kAtomB = kN * 128;  // of B: 16 KB
constexpr int kTileA = 2 * kAtomA, kTileB = 2 * kAtomB;
constexpr int kOffA = 0;                   // A tiles (3)
constexpr int kOffB = kOffA + 3 * kTileA;  // 2 slots x B tile
// Per weight type: the raw rows of a block are one TMA box per slot. A Q4_K block (144 B) is
// 16-byte aligned in its row; a Q6_K block (210 B) is not, so its box starts at the block's
// offset rounded down to 16 bytes and is 240 bytes wide (the block starts (210 b) mod 16 in).
template <bool Q6>
struct Lay {
    static constexpr int kBlockBytes = Q6 ? 210 : 144;
    static constexpr int kRawRow = Q6 ? 240 : 144;
    static constexpr int kRawTile = kM * kRawRow;
    static constexpr int kOffRaw = kOffB + 2 * kTileB;       // 2 slots x 128 rows
    static constexpr int kOffSx = kOffRaw + 2 * kRawTile;    // 2 x 128 token scales
    static constexpr int kOffBar = kOffSx + 2 * kN * 4;      // full[2], a_full, mma_done
    static constexpr int kOffLut = kOffBar + 64;             // Q6_K: scale digits, 256 x u16
    static constexpr int kSmemBytes = kOffLut + (Q6 ? 512 : 0) + 1024;  // + alignment slack
    static constexpr uint32_t kTxBytes = kRawTile + kTileB;  // one block's TMA bytes
    static_assert(kSmemBytes <= 227 * 1024, "shared memory");
};
constexpr uint32_t kTmemCols = 512;               // 3 accumulators x 128 columns, rounded up
constexpr long long kWaitLimit = 1ll << 22;

// Phase timestamps for a timing build (-DBEBELM_QTC_TRACE): clock64 at 4 points of each block
// step, for worker threads 0 and 256 of CTA (0, 0). Compiled out otherwise.
#ifdef BEBELM_QTC_TRACE
__device__ long long g_qtc_trace[2][64][4];
#define QTRACE(slot)                                                                                         \
    do {                                                                                                     \
        if (blockIdx.x == 0 && blockIdx.y == 0 && (threadIdx.x & 255) == 0 && threadIdx.x < kWorkers &&      \
            b < 64)                                                                                          \
            g_qtc_trace[threadIdx.x >> 8][b][slot] = clock64();                                              \
    } while (0)
#else
#define QTRACE(slot) \
    do {             \
    } while (0)
#endif

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {  // 128B swizzle, K-major, SBO 1024, version 1
    return (uint64_t)((addr & 0x3FFFF) >> 4) | ((uint64_t)(16 >> 4) << 16) | ((uint64_t)(1024 >> 4) << 32) |
           (1ull << 46) | (2ull << 61);
}
// kind::i8: D s32 (2 at bit 4), A and B signed 8-bit (1 at bits 7 and 10), both K-major, N, M
constexpr uint32_t kIdesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kN >> 3) << 17) | ((uint32_t)(kM >> 4) << 24);
// kind::f16: D f32 (1 at bit 4), A and B f16 (0 at bits 7 and 10), both K-major, N, M
constexpr uint32_t kIdescF16 = (1u << 4) | ((uint32_t)(kN >> 3) << 17) | ((uint32_t)(kM >> 4) << 24);

// byte offset of (row, k) in a K-major A tile of two 128-byte-swizzled atoms (K 0..127, 128..255):
// inside an atom, 8-row groups of 1024 bytes, the 16-byte chunk index XORed with the row in its group
__device__ __forceinline__ uint32_t swz_a(int row, int k) {
    const uint32_t o = (uint32_t)(row * 128 + (k & 127));
    return (uint32_t)(k >> 7) * kAtomA + (o ^ (((o >> 7) & 7u) << 4));
}

__device__ __forceinline__ bool mbar_try(uint32_t bar, unsigned parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool mbar_wait(uint32_t bar, unsigned parity) {
    for (long long it = 0; it < kWaitLimit; ++it)
        if (mbar_try(bar, parity)) return true;
    return false;
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(dst),
        "l"(map), "r"(x), "r"(y), "r"(bar)
        : "memory");
}
__device__ __forceinline__ void workers_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kWorkers) : "memory"); }

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

// W 32-bit words starting at byte `start` (even) of a 16-byte aligned shared-memory row:
// aligned 16-byte loads, then a word shift by (start % 16) / 4 and a funnel shift by 16 bits
// when start % 4 = 2 (both uniform across the CTA)
template <int W>
__device__ __forceinline__ void load_realigned(const unsigned char* row16, int start, uint32_t* out) {
    uint32_t v[W + 4];
    const uint4* p = reinterpret_cast<const uint4*>(row16 + (start & ~15));
#pragma unroll
    for (int i = 0; i < W / 4 + 1; ++i) {
        const uint4 t = p[i];
        v[4 * i] = t.x, v[4 * i + 1] = t.y, v[4 * i + 2] = t.z, v[4 * i + 3] = t.w;
    }
    const int ws = (start & 15) >> 2;
    const uint32_t bs = (uint32_t)(start & 3) * 8;
#pragma unroll
    for (int i = 0; i < W + 2; ++i) v[i] = (ws & 2) ? v[i + 2] : v[i];
#pragma unroll
    for (int i = 0; i < W + 1; ++i) v[i] = (ws & 1) ? v[i + 1] : v[i];
#pragma unroll
    for (int i = 0; i < W; ++i) out[i] = __funnelshift_r(v[i], v[i + 1], bs);
}

template <bool Q6>
__global__ void __launch_bounds__(kThreads, 1)
    kquant_tc_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_q, size_t n_in,
                  size_t n_out, size_t n_tokens, const float* q8_scales, const int* q8_sums, float* y, int* err) {
    using L = Lay<Q6>;
    extern __shared__ unsigned char smem_raw[];
    unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sb = smem_u32(sm);
    __shared__ uint32_t s_tmem;
    __shared__ int s_fail, s_wfail;  // control warp, workers
    const int tid = threadIdx.x, warp = tid >> 5;
    const size_t r0 = (size_t)blockIdx.x * kM, t0 = (size_t)blockIdx.y * kN;
    const size_t nb = n_in / kQK;
    const uint32_t full0 = sb + L::kOffBar, a_full = full0 + 16, mma_done = full0 + 24;

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    if (tid == kWorkers) {
        for (int i = 0; i < 4; ++i) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(full0 + 8 * i));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        s_fail = s_wfail = 0;
    }
    if constexpr (Q6) {  // balanced base-7 digits (e0, e1, e2) of every int8 scale, each + 3
        if (tid < 256) {
            int r = tid - 128, dg = 0;
            for (int i = 0; i < 3; ++i) {
                const int qt = (r + 3 + 7 * 25) / 7 - 25;  // floor((r + 3) / 7), r >= -171
                dg |= (r - 7 * qt + 3) << (4 * i);
                r = qt;
            }
            reinterpret_cast<unsigned short*>(sm + L::kOffLut)[tid] = (unsigned short)dg;
        }
    }
    tc_before();
    __syncthreads();
    tc_after();
    const uint32_t tmem = s_tmem;

    if (warp == kWorkers / 32) {
        // ---------------- control warp: TMA producer and MMA issuer (lane 0) ----------------
        if ((tid & 31) == 0) {
            auto load = [&](size_t bb) {
                const uint32_t full = full0 + 8 * (uint32_t)(bb & 1), slot = (uint32_t)(bb & 1);
                asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(full), "r"(L::kTxBytes)
                             : "memory");
                tma_load_2d(sb + L::kOffRaw + slot * L::kRawTile, &tm_w, (int)((bb * L::kBlockBytes) & ~size_t(15)), (int)r0,
                            full);
                tma_load_2d(sb + kOffB + slot * kTileB, &tm_q, (int)(bb * kQK), (int)t0, full);
                tma_load_2d(sb + kOffB + slot * kTileB + kAtomB, &tm_q, (int)(bb * kQK + 128), (int)t0, full);
            };
            size_t issued = 0, mmas = 0;
            for (; issued < 2 && issued < nb; ++issued) load(issued);
            for (size_t b = 0; b < nb; ++b) {
                if (!mbar_wait(a_full, (unsigned)(b & 1))) {
                    s_fail = 1;
                    break;
                }
                tc_after();
                const uint32_t bB = sb + kOffB + (uint32_t)(b & 1) * kTileB;
#pragma unroll
                for (int a = 0; a < (Q6 ? 3 : 2); ++a) {
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk) {  // K step: atom kk / 4, 32 bytes at (kk % 4) * 32
                        const uint32_t koff = (uint32_t)(kk & 3) * 32;
                        const uint64_t ad = smem_desc(sb + kOffA + a * kTileA + (kk >> 2) * kAtomA + koff);
                        const uint64_t bd = smem_desc(bB + (kk >> 2) * kAtomB + koff);
                        asm volatile(
                            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                            "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem + a * kN),
                            "l"(ad), "l"(bd), "r"(kIdesc), "r"(kk)
                            : "memory");
                    }
                }
                if constexpr (!Q6) {  // sm: one f16 MMA, K = 16, into the third accumulator (f32)
                    const uint64_t ad = smem_desc(sb + kOffA + 2 * kTileA);
                    const uint64_t bd = smem_desc(sb + kOffA + 2 * kTileA + kAtomA);
                    asm volatile(
                        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem + 2 * kN),
                        "l"(ad), "l"(bd), "r"(kIdescF16), "r"(0)
                        : "memory");
                }
                asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                                 mma_done)
                             : "memory");
                ++mmas;
                if (issued < nb) {  // block b's slot is free once its MMAs are done
                    if (!mbar_wait(mma_done, (unsigned)(b & 1))) {
                        s_fail = 1;
                        break;
                    }
                    load(issued++);
                }
            }
            // nothing of ours may still be in flight when the CTA exits
            for (size_t i = issued >= 2 ? issued - 2 : 0; i < issued; ++i)
                mbar_wait(full0 + 8 * (uint32_t)(i & 1), (unsigned)((i >> 1) & 1));
            if (mmas) mbar_wait(mma_done, (unsigned)((mmas - 1) & 1));
        }
        __syncwarp();
    } else {
        // ---------------- workers: thread (row, quarter) ----------------
        const int row = tid & (kM - 1), quarter = tid >> 7;
        const uint32_t t_lane = tmem + ((uint32_t)(32 * (warp & 3)) << 16) + 32 * quarter;
        const float* sx_src = q8_scales + (t0 + tid) * nb;
        const bool sx_ok = tid < kN && t0 + tid < n_tokens;
        float sx_next = sx_ok && nb ? sx_src[0] : 0.f;
        // Q4_K: the token's 32-wide sub-block sums S_j of the next block (8 ints), for B'
        const int4* sum_src = reinterpret_cast<const int4*>(q8_sums + (t0 + tid) * nb * 8);
        int4 sum_next[2] = {make_int4(0, 0, 0, 0), make_int4(0, 0, 0, 0)};
        if (!Q6 && sx_ok && nb) sum_next[0] = sum_src[0], sum_next[1] = sum_src[1];
        float d = 0.f, dmin = 0.f;  // of the block whose accumulators are read next
        float acc[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) acc[i] = -0.0f;
        for (size_t b = 0; b <= nb; ++b) {
            // block b-1's MMAs done (A free, accumulators complete) and block b's operands landed
            if (tid == 0) {
                bool ok = true;
                if (b >= 1) ok = mbar_wait(mma_done, (unsigned)((b - 1) & 1));
                if (ok && b < nb) ok = mbar_wait(full0 + 8 * (uint32_t)(b & 1), (unsigned)((b >> 1) & 1));
                if (!ok) s_wfail = 1;
            }
            workers_sync();
            QTRACE(0);
            if (*reinterpret_cast<volatile int*>(&s_wfail)) break;  // decided by worker 0 only
            if (b >= 1) mbar_try(mma_done, (unsigned)((b - 1) & 1));  // this thread's own acquire
            if (b < nb) mbar_try(full0 + 8 * (uint32_t)(b & 1), (unsigned)((b >> 1) & 1));
            if (b >= 1) {  // epilogue of block b-1
                tc_after();
                const float* sx = reinterpret_cast<const float*>(sm + L::kOffSx + ((b - 1) & 1) * kN * 4) + 32 * quarter;
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    int a0[16], a1[16], a2[16];
                    tmem_ld16(t_lane + 16 * h, a0);
                    tmem_ld16(t_lane + kN + 16 * h, a1);
                    tmem_ld16(t_lane + 2 * kN + 16 * h, a2);
                    tmem_wait();
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        float v;
                        if constexpr (Q6) {  // s = a0 + 7 a1 + 49 a2; sx * (d * s)
                            const int isum = a0[i] + 7 * a1[i] + 49 * a2[i];
                            v = __fmul_rn(sx[16 * h + i], __fmul_rn(d, __int2float_rn(isum)));
                        } else {  // sd = lo + 8 hi, sm = min; sx * (d * sd - dmin * sm)
                            const int sd = a0[i] + 8 * a1[i];
                            v = __fmul_rn(sx[16 * h + i], __fsub_rn(__fmul_rn(d, __int2float_rn(sd)),
                                                                    __fmul_rn(dmin, __int_as_float(a2[i]))));
                        }
                        acc[16 * h + i] = __fadd_rn(acc[16 * h + i], v);
                    }
                }
                tc_before();
            }
            QTRACE(1);
            if (b == nb) break;
            if constexpr (Q6) {
                // unpack weights 64 quarter .. +63 of `row`: half n = quarter / 2, groups g = 2 (quarter
                // % 2) + gi of 32 weights, each two 16-wide sub-blocks with one int8 scale (layout of
                // dot_q6k_block_q8: ql low/high nibbles, qh 2-bit fields). The block starts o bytes
                // into its 16-byte aligned box row, so its bytes are read with aligned 16-byte loads
                // (conflict-free at the 240-byte row stride) and realigned in registers.
                const int o = (int)((b * L::kBlockBytes) & 15);
                const unsigned char* rowp = sm + L::kOffRaw + (b & 1) * L::kRawTile + row * L::kRawRow;
                d = f16f(*reinterpret_cast<const unsigned short*>(rowp + o + 208));
                const int n = quarter >> 1, hi_nib = quarter & 1;
                uint32_t qlw[16], qhw[8];
                load_realigned<16>(rowp, 64 * n + o, qlw);
                load_realigned<8>(rowp, 128 + 32 * n + o, qhw);
                const signed char* scs = reinterpret_cast<const signed char*>(rowp + o + 192 + 8 * n);
                const unsigned short* lut = reinterpret_cast<const unsigned short*>(sm + L::kOffLut);
#pragma unroll
                for (int gi = 0; gi < 2; ++gi) {
                    const int g = 2 * hi_nib + gi;
#pragma unroll
                    for (int sub = 0; sub < 2; ++sub) {
                        // balanced base-7 digits of the scale: s = e0 + 7 e1 + 49 e2, e_i in [-3, 3]
                        const uint32_t dg = lut[scs[2 * g + sub] + 128];
                        int e[3];
                        uint32_t c[3];
#pragma unroll
                        for (int i = 0; i < 3; ++i) {
                            e[i] = (int)((dg >> (4 * i)) & 15) - 3;
                            c[i] = (uint32_t)(128 - 32 * e[i]) * 0x01010101u;
                        }
                        uint32_t av[3][4];
#pragma unroll
                        for (int w4 = 0; w4 < 4; ++w4) {
                            const uint32_t l = qlw[8 * gi + 4 * sub + w4];
                            const uint32_t nib = hi_nib ? (l >> 4) & 0x0f0f0f0fu : l & 0x0f0f0f0fu;
                            const uint32_t q6 = nib | (((qhw[4 * sub + w4] >> (2 * g)) & 0x03030303u) << 4);
                            // bytewise (q6 - 32) e: q6 e + 128 - 32 e lies in [32, 224] for every byte,
                            // so the 32-bit multiply-add has no carries or borrows between bytes, and
                            // flipping the top bit subtracts the 128 again as an s8
#pragma unroll
                            for (int i = 0; i < 3; ++i) av[i][w4] = (q6 * (uint32_t)e[i] + c[i]) ^ 0x80808080u;
                        }
                        const uint32_t off = swz_a(row, 128 * n + 32 * g + 16 * sub);
#pragma unroll
                        for (int i = 0; i < 3; ++i)
                            *reinterpret_cast<uint4*>(sm + kOffA + i * kTileA + off) =
                                make_uint4(av[i][0], av[i][1], av[i][2], av[i][3]);
                    }
                }
            } else {
                // unpack chunk `quarter` (64 weights: sub-blocks 2q (low nibbles), 2q+1 (high)) of `row`
                const unsigned char* raw = sm + L::kOffRaw + (b & 1) * L::kRawTile + row * L::kRawRow;
                const uint4 sc4 = *reinterpret_cast<const uint4*>(raw);  // d, dmin, scales[0..11]
                d = f16f(sc4.x & 0xffffu);
                dmin = f16f(sc4.x >> 16);
                const uint32_t s0 = sc4.y, s1 = sc4.z, s2 = sc4.w;  // scale bytes 0-3, 4-7, 8-11
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
                        const uint32_t off = swz_a(row, (2 * quarter + h) * 32 + p);
                        *reinterpret_cast<uint4*>(sm + kOffA + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
                        *reinterpret_cast<uint4*>(sm + kOffA + kTileA + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                    }
                }
                // sm = Σ_j m_j S_j as one f16 MMA (K = 16): A' row = the 8 mins twice, B' token =
                // 64 a_j then b_j with S_j = 64 a_j + b_j, b_j in [0, 63]. Every operand is an
                // exact f16 and every partial sum an integer below 2^24, so the f32 result is exact.
                if (quarter == 0) {
                    uint32_t mw[4];
#pragma unroll
                    for (int jj = 0; jj < 8; jj += 2) {
                        uint32_t m2[2];
#pragma unroll
                        for (int u = 0; u < 2; ++u) {
                            const int j = jj + u;
                            m2[u] = j < 4 ? (s1 >> (8 * j)) & 63
                                          : (((s2 >> (8 * (j - 4))) & 0xff) >> 4) | (((s1 >> (8 * (j - 4) + 6)) & 3) << 4);
                        }
                        const __half2 hv = __floats2half2_rn((float)m2[0], (float)m2[1]);
                        mw[jj / 2] = *reinterpret_cast<const uint32_t*>(&hv);
                    }
                    const uint4 mv = make_uint4(mw[0], mw[1], mw[2], mw[3]);
                    *reinterpret_cast<uint4*>(sm + kOffA + 2 * kTileA + swz_a(row, 0)) = mv;
                    *reinterpret_cast<uint4*>(sm + kOffA + 2 * kTileA + swz_a(row, 16)) = mv;
                }
                if (tid < kN) {
                    const int sv[8] = {sum_next[0].x, sum_next[0].y, sum_next[0].z, sum_next[0].w,
                                       sum_next[1].x, sum_next[1].y, sum_next[1].z, sum_next[1].w};
                    uint32_t aw[4], bw[4];
#pragma unroll
                    for (int jj = 0; jj < 8; jj += 2) {
                        const __half2 ha = __floats2half2_rn((float)((sv[jj] >> 6) * 64), (float)((sv[jj + 1] >> 6) * 64));
                        const __half2 hb = __floats2half2_rn((float)(sv[jj] & 63), (float)(sv[jj + 1] & 63));
                        aw[jj / 2] = *reinterpret_cast<const uint32_t*>(&ha);
                        bw[jj / 2] = *reinterpret_cast<const uint32_t*>(&hb);
                    }
                    unsigned char* bp = sm + kOffA + 2 * kTileA + kAtomA;
                    *reinterpret_cast<uint4*>(bp + swz_a(tid, 0)) = make_uint4(aw[0], aw[1], aw[2], aw[3]);
                    *reinterpret_cast<uint4*>(bp + swz_a(tid, 16)) = make_uint4(bw[0], bw[1], bw[2], bw[3]);
                    if (sx_ok && b + 1 < nb) sum_next[0] = sum_src[2 * (b + 1)], sum_next[1] = sum_src[2 * (b + 1) + 1];
                }
            }
            if (tid < kN) {  // this block's token scales for the epilogue; the next block's from memory
                reinterpret_cast<float*>(sm + L::kOffSx + (b & 1) * kN * 4)[tid] = sx_next;
                sx_next = sx_ok && b + 1 < nb ? sx_src[b + 1] : 0.f;
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // A -> tensor core
            workers_sync();
            QTRACE(2);
            if (tid == 0) mbar_arrive(a_full);
        }
        if (!*reinterpret_cast<volatile int*>(&s_wfail)) {
            const size_t r = r0 + row;
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                const size_t t = t0 + 32 * quarter + i;
                if (r < n_out && t < n_tokens) y[t * n_out + r] = acc[i];
            }
        }
    }
    __syncthreads();
    if (tid == 0 && (s_fail || s_wfail)) *reinterpret_cast<volatile int*>(err) = kErrWaitTimeout;
    if (warp == 0) {
        tc_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
    }
}

PFN_cuTensorMapEncodeTiled_v12000 map_encoder() {
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

// a [rows][row_bytes] byte matrix as a 2-D tensor; box = box_x bytes x box_y rows
bool byte_map(CUtensorMap* m, const void* base, size_t row_bytes, size_t rows, uint32_t box_x, uint32_t box_y,
              CUtensorMapSwizzle swizzle) {
    auto enc = map_encoder();
    if (!enc) return false;
    cuuint64_t dims[2] = {(cuuint64_t)row_bytes, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
    cuuint32_t box[2] = {box_x, box_y};
    cuuint32_t estr[2] = {1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

namespace {
template <bool Q6>
cudaError_t launch_tc(const uint8_t* w, size_t n_in, size_t n_out, size_t n_tokens, const int8_t* q8,
                      const float* q8_scales, const int* q8_sums, float* y, int* err, cudaStream_t s) {
    using L = Lay<Q6>;
    const size_t row_bytes = n_in / kQK * L::kBlockBytes;
    // TMA wants 16-byte aligned bases and row strides; rows and tokens must fit the 32-bit
    // coordinates
    if ((reinterpret_cast<uintptr_t>(w) & 15) || (reinterpret_cast<uintptr_t>(q8) & 15) || (row_bytes & 15) ||
        (reinterpret_cast<uintptr_t>(q8_sums) & 15) ||
        n_out >= (1u << 31) || n_tokens >= (1u << 31) || row_bytes >= (1u << 31))
        return cudaErrorNotSupported;
    CUtensorMap tw, tq;
    if (!byte_map(&tw, w, row_bytes, n_out, L::kRawRow, kM, CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !byte_map(&tq, q8, n_in, n_tokens, 128, kN, CU_TENSOR_MAP_SWIZZLE_128B))
        return cudaErrorNotSupported;
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !attr_set[dev]) {
        cudaError_t e =
            cudaFuncSetAttribute(kquant_tc_kernel<Q6>, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kSmemBytes);
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) attr_set[dev] = true;
    }
    const dim3 grid((unsigned)((n_out + kM - 1) / kM), (unsigned)((n_tokens + kN - 1) / kN));
    kquant_tc_kernel<Q6><<<grid, kThreads, L::kSmemBytes, s>>>(tw, tq, n_in, n_out, n_tokens, q8_scales, q8_sums, y,
                                                                err);
    return cudaGetLastError();
}
}  // namespace

cudaError_t launch_kquant_tc(int dtype, const uint8_t* w, size_t n_in, size_t n_out, size_t n_tokens,
                             const int8_t* q8, const float* q8_scales, const int* q8_sums, float* y, int* err,
                             cudaStream_t s) {
    if (dtype == kGgmlQ4K) return launch_tc<false>(w, n_in, n_out, n_tokens, q8, q8_scales, q8_sums, y, err, s);
    if (dtype == kGgmlQ6K) return launch_tc<true>(w, n_in, n_out, n_tokens, q8, q8_scales, q8_sums, y, err, s);
    return cudaErrorNotSupported;
}

}  // namespace bebelm
