// Kernel 2: causal prefill attention on the 5th-generation tensor cores.
//
// Computes, for a chunk of t queries appended after len_before cached positions
// (the reference's `attn_batch`, src/model.rs:232-254, where token i runs
// `attention_decode` over the len_before + i + 1 keys present once its own k/v
// is appended), out[i, h] = Σ_{j <= len_before+i} softmax_j(q_i·k_j * scale) v_j
// with bf16 operands and fp32 accumulation, as a flash-attention loop.
//
// One CTA per (query head, pair of 128-query tiles), one CTA per SM (512 TMEM columns),
// 11 warps in fixed roles:
//   * warp 1 (TMA): the two Q tiles once, then K/V tiles of 128 keys into a 3-stage ring
//     (cp.async.bulk.tensor, 128-byte swizzle, mbarrier complete_tx).
//   * warps 0 and 10 (MMA, one lane each, one per query tile X): S_X = Q_X K^T (4 x
//     tcgen05.mma M=128 N=128 K=16, both operands from shared memory) into TMEM and
//     O_X += P_X V (8 x tcgen05.mma N=64, P read from TMEM, V MN-major from shared memory).
//     MMA issue blocks while the tensor pipe's short queue is full, so each tile has its own
//     issuer and neither waits behind the other's issue.
//   * warps 2-5 / 6-9 (softmax, one TMEM lane = one query row per thread): read S once in
//     64-column chunks, causal mask on the diagonal tile only, online softmax in the exp2
//     domain with a lazy reference max (O and the running sum are rescaled only when a
//     chunk's max exceeds it by 2^8), P to TMEM as bf16, O rescaled in TMEM when needed.
//     Exponentials: the MUFU ex2 for 7 of every 8 pairs of scores, a degree-3 polynomial on
//     the FMA pipe for the 8th, since the MUFU (16 per clock per SM) is the unit that bounds
//     a head_dim-64 tile; packed f32x2 FMAs/adds and a three-input max keep the other
//     instructions from crowding its issue slots.
// Tiles entirely above the diagonal are never visited; the longest tile pairs are scheduled
// first. Every mbarrier wait is bounded: on timeout the CTA records kErrWaitTimeout, waits
// (bounded) for its own copies and MMAs, frees its TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "internal.h"

namespace bebelm {
namespace {

constexpr int kTileQ = 128, kTileK = 128;
constexpr int kTileBytes = kTileQ * kHeadDim * 2;  // 16 KB: 128 rows x 128 B
constexpr long long kWaitLimit = 1ll << 22;

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

// 32 lanes x 64 consecutive columns into 64 registers, wait included (see tmem_ld32).
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float* v) {
    uint32_t r[64];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x64.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32, %33, %34, %35, "
        "%36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, "
        "%57, %58, %59, %60, %61, %62, %63}, [%64];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]),
          "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]),
          "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]),
          "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]),
          "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
}

// 32 lanes x 32 consecutive 32-bit TMEM columns from 32 registers per thread.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t* r) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
        "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
        "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// O_tile += P V with A (= P) read from TMEM.
__device__ __forceinline__ void mma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t idesc,
                                            uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}

__device__ __forceinline__ float ex2(float x) {  // 2^x on the MUFU unit; -inf gives 0
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

#ifndef BEBELM_PF_POLY
#define BEBELM_PF_POLY 2  // of every 16 key pairs, how many take 2^x on the FMA pipe
#endif

// 2^x for two values on the FMA pipe instead of the MUFU unit, so the two units share the
// softmax's exponentials. x is clamped to >= -125 (2^-125 is zero for every later use) and
// split as x = j + f, with j = round(x) from the 1.5*2^23 rounding constant and f in
// [-1/2, 1/2]. 2^f is a degree-3 polynomial, fitted here by least squares to minimise the
// relative error on that interval: max 7.5e-5, far below the bf16 rounding of P. 2^j enters
// the exponent field through one integer multiply-add. Arithmetic is packed f32x2.
__device__ __forceinline__ void exp2_poly2(float& y0, float& y1, float x0, float x1) {
    x0 = fmaxf(x0, -125.0f);
    x1 = fmaxf(x1, -125.0f);
    uint32_t t0, t1, p0, p1;
    asm("{\n\t.reg .b64 x, t, j, f, p, m, c;\n\t"
        "mov.b64 x, {%4, %5};\n\t"
        "mov.b64 m, {%6, %6};\n\t"
        "add.rn.f32x2 t, x, m;\n\t"
        "sub.rn.f32x2 j, t, m;\n\t"
        "sub.rn.f32x2 f, x, j;\n\t"
        "mov.b64 p, {%7, %7};\n\t"
        "mov.b64 c, {%8, %8};\n\t"
        "fma.rn.f32x2 p, p, f, c;\n\t"
        "mov.b64 c, {%9, %9};\n\t"
        "fma.rn.f32x2 p, p, f, c;\n\t"
        "mov.b64 c, {%10, %10};\n\t"
        "fma.rn.f32x2 p, p, f, c;\n\t"
        "mov.b64 {%0, %1}, t;\n\t"
        "mov.b64 {%2, %3}, p;\n\t}"
        : "=r"(t0), "=r"(t1), "=r"(p0), "=r"(p1)
        : "f"(x0), "f"(x1), "f"(12582912.0f), "f"(0.05517161265f), "f"(0.24261112511f), "f"(0.69326096773f),
          "f"(0.99992805719f));
    y0 = __uint_as_float(t0 * (1u << 23) + p0);
    y1 = __uint_as_float(t1 * (1u << 23) + p1);
}

#ifndef BEBELM_PF_ALU_PACK
#define BEBELM_PF_ALU_PACK 0
#endif
// Two non-negative finite floats to a bf16 pair, round to nearest even, on the integer ALU
// (low half = a). Keeps the conversion off the unit that also computes the exponentials.
__device__ __forceinline__ uint32_t pack_bf16_alu(float a, float b) {
    uint32_t ua = __float_as_uint(a), ub = __float_as_uint(b);
    ua += 0x7FFFu + ((ua >> 16) & 1u);
    ub += 0x7FFFu + ((ub >> 16) & 1u);
    return __byte_perm(ua, ub, 0x7632);
}

// max(a, b, c) in one instruction (sm_100)
__device__ __forceinline__ float max3(float a, float b, float c) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}
// (x0, x1) = (v0, v1) * s + (c, c): one packed f32x2 FMA, each lane rounded once as fmaf
__device__ __forceinline__ void ffma2_sc(float& x0, float& x1, float v0, float v1, float s, float c) {
    asm("{\n\t.reg .b64 a, b, c;\n\t"
        "mov.b64 a, {%2, %3};\n\t"
        "mov.b64 b, {%4, %4};\n\t"
        "mov.b64 c, {%5, %5};\n\t"
        "fma.rn.f32x2 c, a, b, c;\n\t"
        "mov.b64 {%0, %1}, c;\n\t}"
        : "=f"(x0), "=f"(x1)
        : "f"(v0), "f"(v1), "f"(s), "f"(c));
}
// (a0, a1) += (b0, b1): one packed f32x2 add
__device__ __forceinline__ void fadd2(float& a0, float& a1, float b0, float b1) {
    asm("{\n\t.reg .b64 a, b;\n\t"
        "mov.b64 a, {%0, %1};\n\t"
        "mov.b64 b, {%2, %3};\n\t"
        "add.rn.f32x2 a, a, b;\n\t"
        "mov.b64 {%0, %1}, a;\n\t}"
        : "+f"(a0), "+f"(a1)
        : "f"(b0), "f"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

#ifdef BEBELM_PREFILL_TRACE
__device__ long long g_trace[16 * 2 * 64];  // [event][tile][j] = clock64, CTA (0,0) only
#define TRACE(ev, j, X)                                                           \
    do {                                                                          \
        if (blockIdx.x == 0 && blockIdx.y == 0 && (j) < 64)                       \
            g_trace[((ev) * 2 + (X)) * 64 + (j)] = clock64();                     \
    } while (0)
// first time / last of several threads, for events more than one site or warp records
#define TRACE_FIRST(ev, j, X)                                                         \
    do {                                                                              \
        if (blockIdx.x == 0 && blockIdx.y == 0 && (j) < 64 && !g_trace[((ev) * 2 + (X)) * 64 + (j)]) \
            g_trace[((ev) * 2 + (X)) * 64 + (j)] = clock64();                         \
    } while (0)
#define TRACE_MAX(ev, j, X)                                                           \
    do {                                                                              \
        if (blockIdx.x == 0 && blockIdx.y == 0 && (j) < 64)                           \
            atomicMax(&g_trace[((ev) * 2 + (X)) * 64 + (j)], (long long)clock64());   \
    } while (0)
#else
#define TRACE_FIRST(ev, j, X) \
    do {                      \
    } while (0)
#define TRACE_MAX(ev, j, X) \
    do {                    \
    } while (0)
#define TRACE(ev, j, X) \
    do {                \
    } while (0)
#endif

// Per-CTA timeline for a timing build (-DBEBELM_PREFILL_CTA_TRACE): %globaltimer at entry, after
// set-up, when tile A's softmax first sees S, at the end of its loop, after its stores, and at
// exit, plus the SM. Compiled out otherwise.
#ifdef BEBELM_PREFILL_CTA_TRACE
__device__ long long g_ctat[2048][8];
#define CTAT(slot)                                                                    \
    do {                                                                              \
        const unsigned cta_ = blockIdx.y * gridDim.x + blockIdx.x;                    \
        if (cta_ < 2048) {                                                            \
            long long t_;                                                             \
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                    \
            g_ctat[cta_][slot] = t_;                                                  \
        }                                                                             \
    } while (0)
#else
#define CTAT(slot) \
    do {           \
    } while (0)
#endif

// ---- roles: warps 0 / 10 MMA for tile A / B, 1 TMA, 2-5 softmax for tile A, 6-9 for tile B ----
constexpr int kWarpMmaB = 10;  // issuer of the second query tile (the first is warp 0)
#ifdef BEBELM_PREFILL_TRACE
constexpr int kWarpWatch = 11;
constexpr int kWarps = 12;  // + a watcher warp that records when each K/V tile lands
#else
constexpr int kWarps = 11;
#endif
constexpr int kCtaThreads = kWarps * 32;
#ifndef BEBELM_PF_STAGES
#define BEBELM_PF_STAGES 3
#endif
constexpr int kStages = BEBELM_PF_STAGES;               // K/V ring depth
constexpr float kRescaleSlack = 8.0f;
                   // log2 headroom before O is rescaled
// shared memory map v2 (offsets from a 1024-byte aligned base)
constexpr int kOff2Q = 0;                               // Q_A, Q_B
constexpr int kOff2K = 2 * kTileBytes;                  // kStages K tiles
constexpr int kOff2V = kOff2K + kStages * kTileBytes;   // kStages V tiles
constexpr int kOff2Bar = kOff2V + kStages * kTileBytes;
// barriers (8 bytes each)
constexpr int kBarQ = 0, kBarK = 1, kBarV = kBarK + kStages, kBarEmpty = kBarV + kStages,
              kBarS = kBarEmpty + kStages, kBarP = kBarS + 2, kBarO = kBarP + 2, kBarC = kBarO + 2,
              kNumBars = kBarC + 2;
constexpr int kSmem2Bytes = kOff2Bar + 8 * kNumBars + 1024;
constexpr int kTmem2Cols = 512;  // S_A [0,128) S_B [128,256) P_A [256,320) P_B [320,384) O_A [384,448) O_B [448,512)
constexpr int kColP = 256, kColO = 384;

__global__ void __launch_bounds__(kCtaThreads, 1)
    prefill_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                   const __grid_constant__ CUtensorMap tm_v, PrefillArgs a) {
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sbase = smem_u32(smem);
    auto bar = [&](int i) -> uint32_t { return sbase + kOff2Bar + 8 * i; };
    __shared__ uint32_t s_tmem;
    __shared__ int s_fail;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n_qt = (a.t + kTileQ - 1) / kTileQ;
    const int n_pairs = (n_qt + 1) / 2;
    // grid (heads, pairs): all heads' longest tile pairs are scheduled before any shorter one
    const int pair = n_pairs - 1 - (int)blockIdx.y;
    const int h = blockIdx.x, kvh = h / (a.n_heads / a.n_kv);
    // tile X in {0 (A), 1 (B)} covers queries [q0_X, q0_X + 128)
    auto n_kt_of = [&](int X) -> int {
        const int q0 = (2 * pair + X) * kTileQ;
        if (q0 >= a.t) return 0;
        return (a.len_before + min(q0 + kTileQ, a.t) - 1) / kTileK + 1;
    };
    const int nkt[2] = {n_kt_of(0), n_kt_of(1)};
    const int nkt_max = max(nkt[0], nkt[1]);
#ifdef BEBELM_PREFILL_CTA_TRACE
    if (tid == 0) {
        CTAT(0);
        unsigned smid;
        asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
        g_ctat[blockIdx.y * gridDim.x + blockIdx.x][6] = smid;
        g_ctat[blockIdx.y * gridDim.x + blockIdx.x][7] = nkt_max;
    }
#endif

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                     "r"(kTmem2Cols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    if (tid == 0) {
        s_fail = 0;
        for (int i = 0; i < kNumBars; ++i)
            mbar_init(bar(i), (i >= kBarP && i < kBarP + 2) || (i >= kBarC && i < kBarC + 2) ? 128
                              : (i >= kBarEmpty && i < kBarEmpty + kStages) ? 2
                                                                                             : 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    // launched as a programmatic dependent: the set-up above overlaps the kernel before (which
    // writes q, k and v); nothing it wrote is read, and nothing is written, before this wait
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (tid == 0) CTAT(1);

    if (warp == 1) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            mbar_expect_tx(bar(kBarQ), 2 * kTileBytes);
            tma_load_3d(sbase + kOff2Q, &tm_q, 0, h, (2 * pair) * kTileQ, bar(kBarQ));
            tma_load_3d(sbase + kOff2Q + kTileBytes, &tm_q, 0, h, (2 * pair + 1) * kTileQ, bar(kBarQ));
            for (int j = 0; j < nkt_max; ++j) {
                const int st = j % kStages;
                if (j >= kStages && !mbar_wait_bounded(bar(kBarEmpty + st), ((j / kStages) - 1) & 1)) {
                    s_fail = 1;
                    break;
                }
                TRACE(5, j, 0);
                mbar_expect_tx(bar(kBarK + st), kTileBytes);
                tma_load_3d(sbase + kOff2K + st * kTileBytes, &tm_k, 0, kvh, j * kTileK, bar(kBarK + st));
                mbar_expect_tx(bar(kBarV + st), kTileBytes);
                tma_load_3d(sbase + kOff2V + st * kTileBytes, &tm_v, 0, kvh, j * kTileK, bar(kBarV + st));
            }
        }
    } else if (warp == 0 || warp == kWarpMmaB) {
        // ---------------- MMA issuers, one per query tile ----------------
        // tcgen05.mma issue blocks while the tensor pipe's short queue is full, so one thread
        // serving both tiles spends its time inside issue and reaches the other tile's ready
        // work late. Here each tile has its own issuer, in the tile's natural order with
        // blocking waits: S(j+1) once K(j+1) is in and softmax has read S(j), then O += P(j) V(j)
        // once P(j) is written. Each issuer commits once per K/V stage to the stage's
        // "empty" barrier (count 2), also for stages past its own last tile.
        if (lane == 0) {
            const int X = warp == 0 ? 0 : 1;
            constexpr uint32_t kIdescS = instr_desc(kTileK, false), kIdescO = instr_desc(kHeadDim, true);
            const uint64_t dq = smem_desc(sbase + kOff2Q + X * kTileBytes, 16, 1024);
            bool ok = mbar_wait_bounded(bar(kBarQ), 0);
            auto issue_s = [&](int j) -> bool {
                if (!mbar_wait_bounded(bar(kBarK + j % kStages), (j / kStages) & 1)) return false;
                if (j > 0 && !mbar_wait_bounded(bar(kBarC + X), (j - 1) & 1)) return false;
                tc_fence_after();
                TRACE(14, j, X);
                const uint64_t dk = smem_desc(sbase + kOff2K + (j % kStages) * kTileBytes, 16, 1024);
#pragma unroll
                for (int k = 0; k < kHeadDim / 16; ++k)  // 16 dims: +32 B in both operands
                    mma_bf16(tmem + 128 * X, dq + (uint64_t)(2 * k), dk + (uint64_t)(2 * k), kIdescS, k > 0);
                mma_commit(bar(kBarS + X));
                TRACE(2, j, X);
                return true;
            };
            auto issue_pv = [&](int j) -> bool {
                if (!mbar_wait_bounded(bar(kBarV + j % kStages), (j / kStages) & 1)) return false;
                if (!mbar_wait_bounded(bar(kBarP + X), j & 1)) return false;
                tc_fence_after();
                TRACE(13, j, X);
                const uint64_t dv = smem_desc(sbase + kOff2V + (j % kStages) * kTileBytes, kTileBytes, 1024);
#pragma unroll
                for (int k = 0; k < kTileK / 16; ++k)  // 16 keys: +8 TMEM columns of P, +2048 B of V
                    mma_bf16_ts(tmem + kColO + 64 * X, tmem + kColP + 64 * X + 8 * k, dv + (uint64_t)(128 * k),
                                kIdescO, (j > 0 || k > 0));
                mma_commit(bar(kBarO + X));
                TRACE(1, j, X);
                return true;
            };
            if (ok && nkt[X] > 0) ok = issue_s(0);
            for (int j = 0; ok && j < nkt_max; ++j) {
                if (j + 1 < nkt[X]) ok = issue_s(j + 1);
                if (ok && j < nkt[X]) ok = issue_pv(j);
                // Past its own last tile, an issuer first waits for use j of the stage to be
                // loaded: the load follows the completion of use j - kStages, so this issuer's
                // arrival cannot count towards an earlier use the other issuer still reads.
                if (ok && j >= nkt[X]) ok = mbar_wait_bounded(bar(kBarK + j % kStages), (j / kStages) & 1);
                if (ok) mma_commit(bar(kBarEmpty + j % kStages));  // fires once this issuer's MMAs so far complete
            }
            if (!ok) s_fail = 1;
        }
#ifdef BEBELM_PREFILL_TRACE
    } else if (warp == kWarpWatch) {
        if (lane == 0)
            for (int j = 0; j < nkt_max && j < 64; ++j) {
                mbar_wait_bounded(bar(kBarK + j % kStages), (j / kStages) & 1);
                TRACE(15, j, 0);
                mbar_wait_bounded(bar(kBarV + j % kStages), (j / kStages) & 1);
                TRACE(15, j, 1);
            }
#endif
    } else if (warp >= 2 && warp < 10) {
        // ---------------- softmax warpgroups ----------------
        // warp w may reach TMEM lanes 32*(w%4) .. +31 only, so each group of four
        // consecutive warps covers the 128 lanes of its tile
        const int X = (warp - 2) >> 2;         // tile
        const int row = 32 * (warp & 3) + lane;  // TMEM lane
        const int qi = (2 * pair + X) * kTileQ + row;
        const long long key_lim = (long long)a.len_before + qi;
        const uint32_t t_s = tmem + ((uint32_t)(32 * (warp & 3)) << 16) + 128 * X;
        const uint32_t t_p = tmem + ((uint32_t)(32 * (warp & 3)) << 16) + kColP + 64 * X;
        const uint32_t t_o = tmem + ((uint32_t)(32 * (warp & 3)) << 16) + kColO + 64 * X;
        float m_used = -INFINITY, l = 0.f;
        bool ok = true;
        for (int j = 0; j < nkt[X]; ++j) {
            ok = __all_sync(0xffffffffu, mbar_wait_bounded(bar(kBarS + X), j & 1));
            if (!ok) break;
            if ((warp & 3) == 0 && lane == 0) TRACE(3, j, X);
            if (warp == 2 && lane == 0 && j == 0) CTAT(2);
            tc_fence_after();
            const long long k0 = (long long)j * kTileK;
            const bool diag = k0 + kTileK - 1 > (long long)a.len_before + (2 * pair + X) * kTileQ;
            // keys of this tile this row may see: columns [0, lim] (all of them off the diagonal)
            const long long lim_ll = key_lim - k0;
            const int lim = diag ? (lim_ll < kTileK - 1 ? (int)lim_ll : kTileK - 1) : kTileK - 1;
            // One pass over S, 64 columns at a time. The reference max m_used moves only when a
            // chunk's max exceeds it by 2^8 (lazy rescale); if the second chunk moves it, the
            // first chunk's P (still in registers) and the running sum are rescaled here and O
            // after the P store. S is read from TMEM exactly once.
            float fo = 1.f;  // factor O must take for this tile
            bool bump = false;
            float ps[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) ps[e] = 0.f;
            uint32_t w[64];  // P of the tile, bf16 pairs
#pragma unroll
            for (int c = 0; c < kTileK; c += 64) {
                const int wo = c / 2;
                float v[64];
                tmem_ld64(t_s + c, v);
                if (c + 64 == kTileK) {  // S_X(j) fully read: the next S may overwrite it
                    tc_fence_before();
                    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar(kBarC + X)) : "memory");
                    if (lane == 0) TRACE_MAX(11, j, X);
                }
                float mxv[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) mxv[e] = -INFINITY;
                if (diag) {
#pragma unroll
                    for (int e = 0; e < 64; ++e)
                        if (c + e <= lim) mxv[e & 7] = fmaxf(mxv[e & 7], v[e]);
                } else {  // three-input max: half an instruction per score
#pragma unroll
                    for (int e = 0; e < 64; e += 2) mxv[(e >> 1) & 7] = max3(mxv[(e >> 1) & 7], v[e], v[e + 1]);
                }
                const float mc = fmaxf(fmaxf(fmaxf(mxv[0], mxv[1]), fmaxf(mxv[2], mxv[3])),
                                       fmaxf(fmaxf(mxv[4], mxv[5]), fmaxf(mxv[6], mxv[7]))) * a.scale_log2;
                if (mc > m_used + kRescaleSlack) {
                    const float f = ex2(m_used - mc);  // 0 while nothing has been seen
                    l *= f;
                    fo *= f;
                    bump = true;
                    if (c > 0) {  // rescale the first chunk's P (bf16 pairs) and its partial sums
#pragma unroll
                        for (int e = 0; e < 32; ++e) {
                            __nv_bfloat162 h = *reinterpret_cast<__nv_bfloat162*>(&w[e]);
                            w[e] = pack_bf16(__low2float(h) * f, __high2float(h) * f);
                        }
#pragma unroll
                        for (int e = 0; e < 8; ++e) ps[e] *= f;
                    }
                    m_used = mc;
                }
                const float neg_m = -m_used;
                if (diag) {
#pragma unroll
                    for (int e = 0; e < 32; ++e) {
                        const float p0 = c + 2 * e <= lim ? ex2(fmaf(v[2 * e], a.scale_log2, neg_m)) : 0.f;
                        const float p1 = c + 2 * e + 1 <= lim ? ex2(fmaf(v[2 * e + 1], a.scale_log2, neg_m)) : 0.f;
                        ps[e & 7] += p0 + p1;
                        w[wo + e] = pack_bf16(p0, p1);
                    }
                } else {
#pragma unroll
                    for (int e = 0; e < 32; ++e) {  // packed f32x2 FMA and add: the MUFU gets more of the issue slots
                        float x0, x1;
                        ffma2_sc(x0, x1, v[2 * e], v[2 * e + 1], a.scale_log2, neg_m);
                        float p0, p1;
                        if (((c / 2 + e) & 15) < BEBELM_PF_POLY) {
                            exp2_poly2(p0, p1, x0, x1);
                        } else {
                            p0 = ex2(x0);
                            p1 = ex2(x1);
                        }
                        fadd2(ps[2 * (e & 3)], ps[2 * (e & 3) + 1], p0, p1);
                        w[wo + e] = BEBELM_PF_ALU_PACK ? pack_bf16_alu(p0, p1) : pack_bf16(p0, p1);
                    }
                }
            }
            const float f = fo;
            if ((warp & 3) == 0 && lane == 0) TRACE(7, j, X);
            // P_X and O_X are read by PV(j-1): wait for it before writing either (S(j) no
            // longer implies it, since S(j) is issued before PV(j-1))
            if (j > 0) {
                ok = __all_sync(0xffffffffu, mbar_wait_bounded(bar(kBarO + X), (j - 1) & 1));
                if (!ok) break;
                tc_fence_after();
            }
            tmem_st32(t_p, w);
            tmem_st32(t_p + 32, w + 32);
            const float psum = ((ps[0] + ps[1]) + (ps[2] + ps[3])) + ((ps[4] + ps[5]) + (ps[6] + ps[7]));
            if (__any_sync(0xffffffffu, bump && j > 0)) {
                // PV(j-1) has completed (waited above) and PV(j) waits for this thread: O_X is stable
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    float o[32];
                    uint32_t w[32];
                    tmem_ld32(t_o + 32 * half, o);
#pragma unroll
                    for (int e = 0; e < 32; ++e) w[e] = __float_as_uint(o[e] * f);
                    tmem_st32(t_o + 32 * half, w);
                }
            }
            l += psum;
            tmem_st_wait();
            if ((warp & 3) == 0 && lane == 0) TRACE(8, j, X);
            tc_fence_before();
            asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar(kBarP + X)) : "memory");
            if ((warp & 3) == 0 && lane == 0) TRACE(4, j, X);
        }
        if (warp == 2 && lane == 0) CTAT(3);
        // epilogue: wait for the last PV, normalise, store
        if (ok && nkt[X] > 0) ok = __all_sync(0xffffffffu, mbar_wait_bounded(bar(kBarO + X), (nkt[X] - 1) & 1));
        if (!ok) s_fail = 1;
        if (nkt[X] > 0 && a.peer_world > 0) {
            // Fused all-gather: the tile's rows go into every rank's landing zone over NVLink as
            // 8-byte words tagged with the step's epoch. A thread holds one row; to make each store
            // instruction cover whole rows (32 lanes x 8 B, one 256-byte run), the rows pass
            // through shared memory half a row at a time (Q_X: its last MMA has completed). Every
            // thread of the group takes part in both barriers, also after a failed wait.
            float o[kHeadDim];
            if (ok) {
                tc_fence_after();
                tmem_ld32(t_o, o);
                tmem_ld32(t_o + 32, o + 32);
            } else {
#pragma unroll
                for (int d = 0; d < kHeadDim; ++d) o[d] = 0.f;
            }
            const float inv = ok && l > 0.f ? 1.f / l : 0.f;
            const unsigned long long e = *reinterpret_cast<const volatile unsigned long long*>(a.peer_epoch) + 1ull;
            const unsigned long long tag = e << 32;
            float* tile = reinterpret_cast<float*>(smem + kOff2Q + X * kTileBytes);  // [128 rows][32], rotated
            const int wq = warp & 3, q0 = (2 * pair + X) * kTileQ;
            const size_t zone0 = ((size_t)(e & 1ull) * a.peer_world + a.peer_rank) * a.peer_slice;
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
#pragma unroll
                for (int c = 0; c < 32; ++c) tile[row * 32 + ((c + row) & 31)] = o[hf * 32 + c] * inv;
                asm volatile("bar.sync %0, 128;" ::"r"(1 + X) : "memory");
                for (int r = 0; r < 32; ++r) {
                    const int rr = wq * 32 + r;
                    if (q0 + rr < a.t) {
                        const unsigned long long word = tag | __float_as_uint(tile[rr * 32 + ((lane + rr) & 31)]);
                        const size_t off = zone0 + ((size_t)(q0 + rr) * a.n_heads + h) * kHeadDim + hf * 32 + lane;
                        for (int w = 0; w < a.peer_world; ++w)
                            asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(a.peer_bufs[w] + off), "l"(word)
                                         : "memory");
                    }
                }
                asm volatile("bar.sync %0, 128;" ::"r"(1 + X) : "memory");
            }
        } else if (ok && nkt[X] > 0) {
            tc_fence_after();
            float o[kHeadDim];
            tmem_ld32(t_o, o);
            tmem_ld32(t_o + 32, o + 32);
            if (qi < a.t) {
                const float inv = l > 0.f ? 1.f / l : 0.f;
                float4* dst = reinterpret_cast<float4*>(a.out + ((size_t)qi * a.n_heads + h) * kHeadDim);
#pragma unroll
                for (int d = 0; d < kHeadDim; d += 4)
                    dst[d / 4] = make_float4(o[d] * inv, o[d + 1] * inv, o[d + 2] * inv, o[d + 3] * inv);
            }
        }
        if (warp == 2 && lane == 0) CTAT(4);
    }

    tc_fence_before();
    __syncthreads();
    if (s_fail && tid == 0) {
        *reinterpret_cast<volatile int*>(a.err) = kErrWaitTimeout;
        // let copies and MMAs this CTA started land (bounded) before its memory goes away
        for (int st = 0; st < kStages; ++st) {
            mbar_wait_bounded(bar(kBarK + st), 0);
            mbar_wait_bounded(bar(kBarV + st), 0);
        }
        for (int X = 0; X < 2; ++X) mbar_wait_bounded(bar(kBarO + X), 0);
    }
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmem2Cols));
        if (lane == 0) CTAT(5);
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

bool prefill_make_maps(const PrefillArgs& a, PrefillMaps* m) {
    const long long s_total = (long long)a.len_before + a.t;
    static_assert(sizeof(CUtensorMap) == sizeof(m->q), "tensor map size");
    return make_map(reinterpret_cast<CUtensorMap*>(m->q), a.q, a.n_heads, a.t) &&
           make_map(reinterpret_cast<CUtensorMap*>(m->k), a.k, a.n_kv, s_total) &&
           make_map(reinterpret_cast<CUtensorMap*>(m->v), a.v, a.n_kv, s_total);
}

cudaError_t launch_prefill(const PrefillArgs& a, const PrefillMaps& m, cudaStream_t s) {
    if (a.t <= 0) return cudaSuccess;
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem2Bytes);
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) attr_set[dev] = true;
    }
    const int n_qt = (a.t + kTileQ - 1) / kTileQ;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)a.n_heads, (unsigned)((n_qt + 1) / 2));
    cfg.blockDim = dim3(kCtaThreads);
    cfg.dynamicSmemBytes = (size_t)kSmem2Bytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, prefill_kernel, *reinterpret_cast<const CUtensorMap*>(m.q),
                              *reinterpret_cast<const CUtensorMap*>(m.k), *reinterpret_cast<const CUtensorMap*>(m.v), a);
}

}  // namespace bebelm
