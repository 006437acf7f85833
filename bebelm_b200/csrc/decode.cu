// Kernel 3: split-K single-query GQA decode over the paged KV cache, with the
// combine of the splits fused into the last CTA of each (sequence, kv head),
// and — for a decode step — the q/k RMSNorm + RoPE and the KV append fused in.
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
// Fused step (src/model.rs:440-451): with q_raw set, each CTA norms and ropes
// its own query heads (norm_rope_heads, src/model.rs:600-608, same arithmetic as
// norm_rope.cu); the CTA whose pages hold the appended slot norms and ropes the
// new k, stores k and v into the cache, and uses them for that row directly.
//
// Data movement: one thread issues 1-D bulk TMA copies (cp.async.bulk) of a
// page's K rows (16 KB) and V rows (16 KB) for this kv head into a 3-stage
// shared-memory ring, completed on an mbarrier, plus L2 prefetches of the next
// pages. A stage is handed back as soon as all 4 warps hold their rows in
// registers; the last warp to release it issues the refill, so no CTA-wide
// barrier sits in the streaming loop. Every wait is bounded: on timeout the CTA
// records kErrWaitTimeout, lets its own copies land (bounded again) and returns.
//
// Programmatic dependent launch: before griddepcontrol.wait a CTA only loads its
// page-table slice, initialises barriers and starts copies of pages that hold
// no slot >= dep_slot (the slots the predecessor may still be writing); all
// inputs and every global store come after the wait. The kernel triggers its
// dependents when its streaming loop ends, so the next step's prologue overlaps
// this step's merge.
//
// Compute mapping (128 threads, 4 warps): warp w owns rows 16w..16w+15 of each
// 64-row page; lane = 4*j + p handles rows 16w+j and 16w+8+j and the 16 dims
// of float4 chunks c_i = ((i+j)&3)*4 + p, i = 0..3. The rotation by j makes
// every float4 shared-memory read conflict-free and lets each lane keep its q
// slice in registers; the 4 lanes of a row reduce the dot with two xor
// shuffles (identical result on all 4 lanes).
#include <algorithm>

#include "internal.h"

namespace bebelm {
namespace {

#ifndef BEBELM_DECODE_STAGES
#define BEBELM_DECODE_STAGES 3
#endif
#ifndef BEBELM_DECODE_PREFETCH
#define BEBELM_DECODE_PREFETCH 2
#endif
constexpr int kStages = BEBELM_DECODE_STAGES;
constexpr int kThreads = 128;
constexpr int kRingBytes = kStages * 2 * kPageRowFloats * 4;  // the shared-memory ring: 3 fp32 pages of K + V
constexpr long long kWaitLimit = 1ll << 22;          // try_wait polls before giving up
constexpr int kPrefetch = BEBELM_DECODE_PREFETCH;     // pages prefetched into L2 beyond the ring
#ifndef BEBELM_DECODE_EARLY_PREFETCH
#define BEBELM_DECODE_EARLY_PREFETCH 2
#endif
// pages beyond the ring prefetched into L2 before griddepcontrol.wait: they load while the
// previous step's grid finishes its merge (more of them slow that merge down: 2, 5, 8 and 11
// gave 27.4, 28.6, 29.9 and 30.9 us per config-3 step, 0 and 1 gave 29.9 and 29.4)
constexpr int kEarlyPrefetch = BEBELM_DECODE_EARLY_PREFETCH;
constexpr int kMaxPagesPerSplit = kDecodeMaxPagesPerSplit;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
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

__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, unsigned parity, long long limit = kWaitLimit) {
    for (long long it = 0; it < limit; ++it)
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

__device__ __forceinline__ void bulk_prefetch_l2(const void* src, unsigned bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ unsigned atomic_add_acq_rel_gpu(unsigned* p, unsigned v) {
    unsigned old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

__device__ __forceinline__ float fast_exp2(float x) { return exp2f(x); }

// (c0, c1) += (a0, a1) * (b0, b1). PACKED: one f32x2 FMA instruction (two fp32 FMAs, each
// rounded once), which pays where the loop is short of issue slots (the bf16 cache moves half
// the bytes per FMA); otherwise two scalar FMAs.
template <bool PACKED>
__device__ __forceinline__ void fma2(float& c0, float& c1, float a0, float a1, float b0, float b1) {
    if (PACKED) {
        asm("{\n\t.reg .b64 a, b, c;\n\t"
        "mov.b64 a, {%2, %3};\n\t"
        "mov.b64 b, {%4, %5};\n\t"
        "mov.b64 c, {%0, %1};\n\t"
        "fma.rn.f32x2 c, a, b, c;\n\t"
        "mov.b64 {%0, %1}, c;\n\t}"
        : "+f"(c0), "+f"(c1)
        : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
    } else {
        c0 = fmaf(a0, b0, c0);
        c1 = fmaf(a1, b1, c1);
    }
}

// This step's epoch for the fused all-gather: one more than the group's device word (read after
// griddepcontrol.wait: the previous step's gather kernel advanced it). Its parity picks the
// landing buffer; its low 32 bits tag every element written there.
__device__ __forceinline__ unsigned long long peer_step(const DecodeArgs& a) {
    return *reinterpret_cast<const volatile unsigned long long*>(a.peer_epoch) + 1ull;
}

// Final output element `idx` (head*64 + d) of sequence `seq`: to `out`, or, for the fused
// all-gather, into this rank's slice of every rank's landing zone as one 8-byte word (the
// step's tag above the float's bits), stored over NVLink: a reader knows the value has arrived
// when it sees the tag, so no fence or flag follows the stores.
__device__ __forceinline__ void emit_out(const DecodeArgs& a, int seq, size_t idx, float v, unsigned long long pe) {
    if (a.peer_world > 0) {
        const size_t off = ((size_t)(pe & 1ull) * a.peer_world + a.peer_rank) * a.n_heads * kHeadDim + idx;
        const unsigned long long word = (pe << 32) | __float_as_uint(v);
        for (int w = 0; w < a.peer_world; ++w)
            asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(a.peer_bufs[w] + off), "l"(word) : "memory");
    } else {
        a.out[(size_t)seq * a.n_heads * kHeadDim + idx] = v;
    }
}

// Step plans: every CTA counts itself done once it has used the step counter; the last CTA
// of the grid advances the counter for the next step (which reads it after its
// griddepcontrol.wait, i.e. after this grid has completed).
__device__ __forceinline__ void step_done(const DecodeArgs& a) {
    if (!a.step || threadIdx.x != 0) return;
    const unsigned total = gridDim.x * gridDim.y;
    if (atomicAdd(&a.step->done, 1u) == total - 1) {
        a.step->done = 0u;
        a.step->n += 1ull;
    }
}

// One head of 64 at `pos`, one warp: lane i returns elements i and i+32 after
// rmsnorm (f64 sum of f32 squares, IEEE divide/sqrt, unfused products) and NEOX
// RoPE with the iterative angle — the arithmetic of norm_rope.cu.
__device__ __forceinline__ void warp_norm_rope64(const float* x, const float* gain, long long pos, float ts,
                                                 float eps, int lane, float& y0, float& y1) {
    float a = x[lane], b = x[lane + 32];
    double ss = (double)__fmul_rn(a, a) + (double)__fmul_rn(b, b);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float mean = __double2float_rn(ss / 64.0);
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
    a = __fmul_rn(__fmul_rn(a, scale), gain[lane]);
    b = __fmul_rn(__fmul_rn(b, scale), gain[lane + 32]);
    float theta = __ll2float_rn(pos);
    for (int t = 0; t < lane; ++t) theta = __fmul_rn(theta, ts);
    const float sn = sinf(theta), cs = cosf(theta);
    y0 = __fsub_rn(__fmul_rn(a, cs), __fmul_rn(b, sn));
    y1 = __fadd_rn(__fmul_rn(a, sn), __fmul_rn(b, cs));
}

// Per-CTA timeline for a timing build (-DBEBELM_DECODE_TRACE): %globaltimer at entry, after
// griddepcontrol.wait, first stage landed, streaming done, exit. Compiled out otherwise.
#ifdef BEBELM_DECODE_TRACE
__device__ long long g_dtrace[4][1024 * 8];  // by the first sequence's position mod 4
#define DTRACE(slot)                                                                          \
    do {                                                                                      \
        const unsigned cta_ = blockIdx.y * gridDim.x + blockIdx.x;                             \
        if (threadIdx.x == 0 && cta_ < 1024) {                                                 \
            long long t_;                                                                     \
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                            \
            g_dtrace[a.one.pos & 3][cta_ * 8 + (slot)] = t_;                                  \
        }                                                                                     \
    } while (0)
#else
#define DTRACE(slot) \
    do {             \
    } while (0)
#endif

template <int HPC, int KT>
__device__ __forceinline__ void decode_body(DecodeArgs a) {
    // KT: the cache's element type. bf16 and fp8 (e4m3) rows take a half and a quarter of the
    // bytes, so the same ring holds two and four times the stages; BF: a narrow type, whose
    // loop is short of issue slots rather than of bytes (packed FMAs)
    constexpr bool BF = KT != kElemF32;
    constexpr int ES = KT == kElemF32 ? 4 : KT == kElemBF16 ? 2 : 1;
    constexpr int ROWB = kPageRowFloats * ES;  // one kv head of one page
    constexpr int SB = 2 * ROWB;               // a stage: its K rows and V rows
    constexpr int NST = kRingBytes / SB;
    extern __shared__ __align__(128) unsigned char smem[];
    unsigned char* stages = smem;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kRingBytes);
    __shared__ float s_m[4][HPC], s_l[4][HPC];
    __shared__ int s_release[NST];
    __shared__ int s_failed, s_last;
    __shared__ int s_issued;  // pages whose copies have been issued (the stream's cleanup waits for these)
    __shared__ uint64_t s_never;  // test hook: a barrier that nothing arrives on
    __shared__ int s_phys[kMaxPagesPerSplit];
    __shared__ __align__(16) float s_q[HPC][kHeadDim];
    __shared__ __align__(16) float s_knew[kHeadDim], s_vnew[kHeadDim];
    __shared__ float s_L[HPC];

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int j = lane >> 2, p = lane & 3;
    const int NY = a.n_kv * a.n_sub;
    const int y = blockIdx.y;
    const int kvh = y / a.n_sub, sub = y % a.n_sub;
    const int h0 = kvh * a.group + sub * HPC;

    // which sequence owns this split
    const int gsplit = blockIdx.x;
    DTRACE(0);
    int lo = 0, hi = a.n_seqs - 1;
    while (lo < hi) {
        int mid = (lo + hi + 1) >> 1;
        if (a.seqs[mid].split0 <= gsplit) lo = mid; else hi = mid - 1;
    }
    const int seq = lo;
    DecodeSeq S = a.n_seqs == 1 ? a.one : a.seqs[seq];
    if (a.step) {
        // device-driven step: the window follows from the steps already taken, which this
        // plan's previous step counted when it finished. Unless that step is known to be
        // complete already (step_prewait), the counter is read after the wait and no page is
        // copied before it; otherwise nothing the predecessor writes is in this layer's window.
        if (!a.step_prewait) grid_dep_wait();
        const long long n = (long long)*reinterpret_cast<volatile unsigned long long*>(&a.step->n);
        S.new_slot = a.step_slot0 + n;
        S.pos = a.step_pos0 + n;
        S.len = a.step_len0 + n + 1 < a.step_window ? a.step_len0 + n + 1 : a.step_window;
        S.base = S.new_slot + 1 - S.len;
        S.dep_slot = a.step_prewait ? LLONG_MAX : -1;
    }
    const int split = gsplit - S.split0;
    const long long first_page = S.base >> 6;
    const long long last_page = S.len > 0 ? (S.base + S.len - 1) >> 6 : first_page - 1;
    const long long p0 = first_page + (long long)split * a.pages_per_split;
    long long p1 = p0 + a.pages_per_split;
    if (p1 > last_page + 1) p1 = last_page + 1;
    const int np = p1 > p0 ? (int)(p1 - p0) : 0;
    // pages [0, n_early) hold no slot the predecessor may still write
    const long long dep_page = S.dep_slot >> 6;
    const int n_early = dep_page <= p0 ? 0 : (int)min((long long)np, dep_page - p0);

    // this CTA's query heads, normed + roped here for a fused step, and the appended token's
    // k (normed + roped) and v if its slot is in our pages: computed before griddepcontrol.wait
    // when the host saw that the inputs were complete before the predecessor began (early_inputs)
    const bool has_new = S.new_slot >= 0 && (S.new_slot >> 6) >= p0 && (S.new_slot >> 6) < p1 && sub == 0;
    const bool own_new = S.new_slot >= 0 && (S.new_slot >> 6) >= p0 && (S.new_slot >> 6) < p1;
    auto read_inputs = [&]() {
        if (warp < HPC) {
            const int h = h0 + warp;
            if (a.q_raw) {
                float y0, y1;
                warp_norm_rope64(a.q_raw + ((size_t)seq * a.n_heads + h) * kHeadDim, a.q_gain, S.pos,
                                 a.theta_scale, a.eps, lane, y0, y1);
                s_q[warp][lane] = y0;
                s_q[warp][lane + 32] = y1;
            } else {
                const float* qs = a.q + ((size_t)seq * a.n_heads + h) * kHeadDim;
                s_q[warp][lane] = qs[lane];
                s_q[warp][lane + 32] = qs[lane + 32];
            }
        }
        if (own_new && warp == HPC % 4) {
            const float* kr = a.k_new + ((size_t)seq * a.n_kv + kvh) * kHeadDim;
            const float* vr = a.v_new + ((size_t)seq * a.n_kv + kvh) * kHeadDim;
            float y0, y1;
            warp_norm_rope64(kr, a.k_gain, S.pos, a.theta_scale, a.eps, lane, y0, y1);
            float w0 = vr[lane], w1 = vr[lane + 32];
            if (BF) {  // this step uses exactly what the cache will hold
                y0 = round_to_kind(y0, KT);
                y1 = round_to_kind(y1, KT);
                w0 = round_to_kind(w0, KT);
                w1 = round_to_kind(w1, KT);
            }
            s_knew[lane] = y0;
            s_knew[lane + 32] = y1;
            s_vnew[lane] = w0;
            s_vnew[lane + 32] = w1;
        }
    };
    const bool early = a.early_inputs && !a.step;

    // page-table slice (written by the host, never by a kernel): its loads are started first, so
    // that with early inputs their latency overlaps the norm and RoPE of the step's inputs
    static_assert(kMaxPagesPerSplit <= 2 * kThreads, "page-table slice: two entries per thread");
    int ph[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
        const int i = tid + u * kThreads;
        ph[u] = i < np ? S.table[(int)((p0 + i) % S.cap)] : 0;
    }
    if (early) read_inputs();
#pragma unroll
    for (int u = 0; u < 2; ++u)
        if (tid + u * kThreads < np) s_phys[tid + u * kThreads] = ph[u];
    __syncthreads();
    auto page_src = [&](int i) -> const char* {
        return a.pv.base + (size_t)s_phys[i] * a.pv.page_bytes + a.pv.layer_off + (size_t)kvh * ROWB;
    };
    auto issue = [&](int i) {
        const int st = i % NST;
        const char* kp = page_src(i);
        unsigned char* dk = stages + (size_t)st * SB;
        mbar_expect_tx(&full[st], SB);
        bulk_g2s(dk, kp, ROWB, &full[st]);
        bulk_g2s(dk + ROWB, kp + a.pv.block_bytes, ROWB, &full[st]);
    };
    auto prefetch = [&](int i) {
        const char* kp = page_src(i);
        bulk_prefetch_l2(kp, ROWB);
        bulk_prefetch_l2(kp + a.pv.block_bytes, ROWB);
    };

    const int n_first = min(NST, np);
    if (tid == 0) {
        for (int s = 0; s < NST; ++s) {
            mbar_init(&full[s], 1);
            s_release[s] = 0;
        }
        s_failed = 0;
        s_issued = 0;
        mbar_init(&s_never, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        for (int i = 0; i < n_first && i < n_early; ++i) issue(i);
        s_issued = max(0, min(n_first, n_early));
        for (int i = NST; i < NST + kEarlyPrefetch && i < n_early; ++i) prefetch(i);
    }


    // ---- everything below may read what the predecessor wrote --------------
    grid_dep_wait();
    DTRACE(1);
    const unsigned long long pe = a.peer_world > 0 ? peer_step(a) : 0ull;
    if (tid == 0)
        for (int i = n_early; i < n_first; ++i) issue(i);
    if (tid == 0) s_issued = n_first;
    if (!early) read_inputs();
    if (has_new && warp == HPC % 4) {  // one CTA per kv head writes the cache (the warp that computed it)
        const int i = (int)((S.new_slot >> 6) - p0);
        char* kd = a.pv.base + (size_t)s_phys[i] * a.pv.page_bytes + a.pv.layer_off + (size_t)kvh * ROWB +
                   (size_t)(S.new_slot & 63) * kHeadDim * ES;
        char* vd = kd + a.pv.block_bytes;
        const float y0 = s_knew[lane], y1 = s_knew[lane + 32], w0 = s_vnew[lane], w1 = s_vnew[lane + 32];
        if (KT == kElemBF16) {
            reinterpret_cast<__nv_bfloat16*>(kd)[lane] = __float2bfloat16_rn(y0);
            reinterpret_cast<__nv_bfloat16*>(kd)[lane + 32] = __float2bfloat16_rn(y1);
            reinterpret_cast<__nv_bfloat16*>(vd)[lane] = __float2bfloat16_rn(w0);
            reinterpret_cast<__nv_bfloat16*>(vd)[lane + 32] = __float2bfloat16_rn(w1);
        } else if (KT == kElemFP8) {  // the values are e4m3-exact already
            reinterpret_cast<unsigned char*>(kd)[lane] = float_to_fp8(y0);
            reinterpret_cast<unsigned char*>(kd)[lane + 32] = float_to_fp8(y1);
            reinterpret_cast<unsigned char*>(vd)[lane] = float_to_fp8(w0);
            reinterpret_cast<unsigned char*>(vd)[lane + 32] = float_to_fp8(w1);
        } else {
            reinterpret_cast<float*>(kd)[lane] = y0;
            reinterpret_cast<float*>(kd)[lane + 32] = y1;
            reinterpret_cast<float*>(vd)[lane] = w0;
            reinterpret_cast<float*>(vd)[lane + 32] = w1;
        }
    }
    __syncthreads();

    // q slice of this lane, pre-rotated so register index i pairs with chunk c_i
    int c[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) c[i] = (((i + j) & 3) << 2) + p;
    float4 qr[HPC][4];
#pragma unroll
    for (int h = 0; h < HPC; ++h)
#pragma unroll
        for (int i = 0; i < 4; ++i) qr[h][i] = reinterpret_cast<const float4*>(s_q[h])[c[i]];
    float acc[HPC][16];
    float m[HPC], l[HPC];
#pragma unroll
    for (int h = 0; h < HPC; ++h) {
        m[h] = -INFINITY;
        l[h] = 0.f;
#pragma unroll
        for (int e = 0; e < 16; ++e) acc[h][e] = 0.f;
    }
    if (tid == 0)
        for (int i = max(n_early, NST); i < NST + kEarlyPrefetch && i < np; ++i) prefetch(i);

    const long long win_lo = S.base, win_hi = S.base + S.len;
    const long long new_slot = own_new ? S.new_slot : -1;
    for (int i = 0; i < np; ++i) {
        const int st = i % NST;
        // (test hook: CTA (0, 0) first waits, with a short limit, on a barrier nothing completes)
        const bool expire = a.expire_wait && i == 0 && blockIdx.x == 0 && blockIdx.y == 0;
        const bool ok = __all_sync(0xffffffffu, expire ? mbar_wait_bounded(&s_never, 0u, kWaitLimit >> 8)
                                                       : mbar_wait_bounded(&full[st], (unsigned)((i / NST) & 1)));
        if (i == 0) DTRACE(2);
        if (!ok) {
            if (lane == 0) {
                *reinterpret_cast<volatile int*>(a.err) = kErrWaitTimeout;
                atomicExch(&s_failed, 1);
            }
            break;
        }
        // 4 elements of chunk c of row r, as floats (16 B of fp32, 8 B of bf16, 4 B of fp8)
        const unsigned char* Kst = stages + (size_t)st * SB;
        const unsigned char* Vst = Kst + ROWB;
        auto ld4 = [&](const unsigned char* base, int idx) -> float4 {
            if (KT == kElemFP8) return fp8x4_to_float4(reinterpret_cast<const uint32_t*>(base)[idx]);
            if (KT == kElemBF16) {
                const uint2 u = reinterpret_cast<const uint2*>(base)[idx];
                return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u),
                                   __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xffff0000u));
            }
            return reinterpret_cast<const float4*>(base)[idx];
        };
        const long long slot0 = (p0 + i) << 6;
        // both rows of K and V into registers, then hand the stage back at once
        float4 kk[2][4], vv[2][4];
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const int row = 16 * warp + 8 * r + j;
            if (slot0 + row == new_slot) {  // the appended token: take it from this CTA's own copy
#pragma unroll
                for (int ii = 0; ii < 4; ++ii) {
                    kk[r][ii] = reinterpret_cast<const float4*>(s_knew)[c[ii]];
                    vv[r][ii] = reinterpret_cast<const float4*>(s_vnew)[c[ii]];
                }
            } else {
#pragma unroll
                for (int ii = 0; ii < 4; ++ii) {
                    kk[r][ii] = ld4(Kst, row * 16 + c[ii]);
                    vv[r][ii] = ld4(Vst, row * 16 + c[ii]);
                }
            }
        }
        __syncwarp();
        if (lane == 0) {
            if (atomicAdd(&s_release[st], 1) == 3) {  // last of the 4 warps refills the stage
                s_release[st] = 0;
                if (i + NST < np) {
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    issue(i + NST);
                    s_issued = i + NST + 1;
                    if (i + NST + kPrefetch < np) prefetch(i + NST + kPrefetch);
                }
            }
        }
        float s[2][HPC];
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const long long slot = slot0 + 16 * warp + 8 * r + j;
            const bool valid = slot >= win_lo && slot < win_hi;
#pragma unroll
            for (int h = 0; h < HPC; ++h) {
                float d0 = 0.f, d1 = 0.f;  // even and odd dims, summed at the end
#pragma unroll
                for (int ii = 0; ii < 4; ++ii) {
                    fma2<BF>(d0, d1, qr[h][ii].x, qr[h][ii].y, kk[r][ii].x, kk[r][ii].y);
                    fma2<BF>(d0, d1, qr[h][ii].z, qr[h][ii].w, kk[r][ii].z, kk[r][ii].w);
                }
                float d = d0 + d1;
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
#pragma unroll
            for (int h = 0; h < HPC; ++h) {
                const float w = pr[r][h];
#pragma unroll
                for (int ii = 0; ii < 4; ++ii) {
                    fma2<BF>(acc[h][4 * ii + 0], acc[h][4 * ii + 1], w, w, vv[r][ii].x, vv[r][ii].y);
                    fma2<BF>(acc[h][4 * ii + 2], acc[h][4 * ii + 3], w, w, vv[r][ii].z, vv[r][ii].w);
                }
            }
        }
    }
    // the next launch may start its prologue now (it writes nothing before its own wait)
    DTRACE(3);
    grid_dep_launch();
    __syncthreads();
    if (s_failed) {
        // a wait gave up: let our own copies still in flight land (bounded), then leave
        if (tid == 0) {
            const int n_iss = s_issued;
            for (int k = 0; k < NST && k < n_iss; ++k) {  // the last issued use of stage k
                const int last = ((n_iss - 1 - k) / NST) * NST + k;
                mbar_wait_bounded(&full[k], (unsigned)((last / NST) & 1));
            }
        }
        step_done(a);
        return;
    }

    // ---- merge the 8 row-lanes x 4 warps of this CTA ----------------------
#pragma unroll
    for (int h = 0; h < HPC; ++h) {
        l[h] += __shfl_xor_sync(0xffffffffu, l[h], 4);
        l[h] += __shfl_xor_sync(0xffffffffu, l[h], 8);
        l[h] += __shfl_xor_sync(0xffffffffu, l[h], 16);
    }
    float* red = reinterpret_cast<float*>(stages);  // [4 warps][8 j][HPC][64]; every copy has landed and been read
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
            emit_out(a, seq, (size_t)(h0 + h) * kHeadDim + d, L > 0.f ? A / L : 0.f, pe);
        } else {
            const size_t pi = ((size_t)gsplit * NY + y) * HPC + h;
            a.part_acc[pi * kHeadDim + d] = A;
            if (d == 0) {
                a.part_ml[pi * 2 + 0] = M;
                a.part_ml[pi * 2 + 1] = L;
            }
        }
    }
    if (single) {
        step_done(a);
        DTRACE(4);
        return;
    }

    // ---- last CTA of this (sequence, kv head) merges the splits ----------
    DTRACE(5);
    __syncthreads();  // every partial of this CTA is stored before thread 0 releases it
    if (tid == 0) {
        unsigned* ctr = a.counters + (size_t)seq * NY + y;
        const unsigned prev = atomic_add_acq_rel_gpu(ctr, 1u);
        s_last = (prev == (unsigned)(S.n_splits - 1));
        if (s_last) *ctr = 0u;  // ready for the next launch
    }
    __syncthreads();
    DTRACE(6);
    if (!s_last) {
        DTRACE(4);
        step_done(a);
        return;
    }
    const int ns = S.n_splits;
    constexpr int kVec = HPC * kHeadDim / 4;  // float4s per split record
    constexpr int G = kThreads / kVec;        // thread groups, each a stride of the splits
    const int ml_stride = (ns * HPC + 3) & ~3;  // keeps sm_acc 16-byte aligned for float4 stores
    float* sm_m = red;                          // [ns][HPC] split maxima, then rescale factors
    float* sm_l = red + ml_stride;              // [ns][HPC]
    float* sm_acc = sm_l + ml_stride;           // [G][HPC*64]
    const bool active = tid < G * kVec;
    const int f = tid % kVec, g0 = tid / kVec;
    const int hh = (f * 4) / kHeadDim;
    const float4* src = reinterpret_cast<const float4*>(a.part_acc) + ((size_t)S.split0 * NY + y) * kVec + f;
    const size_t stride = (size_t)NY * kVec;
    // one round of loads: split maxima/sums and this thread's first kRound partial vectors
    // (kRound * G splits: 40 with 128 threads and 4 heads, enough for a 32k window's 37 splits)
    constexpr int kRound = 20;
    float4 x[kRound];
#pragma unroll
    for (int u = 0; u < kRound; ++u) {
        const int k = g0 + u * G;
        x[u] = active && k < ns ? __ldcg(src + (size_t)k * stride) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    for (int t = tid; t < ns * HPC; t += kThreads) {
        const size_t pi = ((size_t)(S.split0 + t / HPC) * NY + y) * HPC + (t % HPC);
        sm_m[t] = __ldcg(a.part_ml + pi * 2);
        sm_l[t] = __ldcg(a.part_ml + pi * 2 + 1);
    }
    __syncthreads();
    DTRACE(7);
    if (warp < HPC) {  // warp h: the splits' maximum and rescaled sum of head h, lanes over splits
        const int h = warp;
        float M = -INFINITY;
        for (int k = lane; k < ns; k += 32) M = fmaxf(M, sm_m[k * HPC + h]);
#pragma unroll
        for (int o2 = 16; o2 > 0; o2 >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o2));
        float L = 0.f;
        for (int k = lane; k < ns; k += 32) {
            const float fk = M == -INFINITY ? 0.f : fast_exp2(sm_m[k * HPC + h] - M);
            sm_m[k * HPC + h] = fk;  // now the rescale factor of split k
            L = fmaf(fk, sm_l[k * HPC + h], L);
        }
#pragma unroll
        for (int o2 = 16; o2 > 0; o2 >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o2);
        if (lane == 0) s_L[h] = L;
    }
    __syncthreads();
    if (active) {
        float4 A = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int k0 = g0; k0 < ns; k0 += kRound * G) {
            if (k0 != g0) {  // more splits than one round holds
#pragma unroll
                for (int u = 0; u < kRound; ++u) {
                    const int k = k0 + u * G;
                    x[u] = k < ns ? __ldcg(src + (size_t)k * stride) : make_float4(0.f, 0.f, 0.f, 0.f);
                }
            }
#pragma unroll
            for (int u = 0; u < kRound; ++u) {
                const int k = k0 + u * G;
                const float fk = k < ns ? sm_m[k * HPC + hh] : 0.f;
                A.x = fmaf(fk, x[u].x, A.x);
                A.y = fmaf(fk, x[u].y, A.y);
                A.z = fmaf(fk, x[u].z, A.z);
                A.w = fmaf(fk, x[u].w, A.w);
            }
        }
        reinterpret_cast<float4*>(sm_acc)[g0 * kVec + f] = A;
    }
    __syncthreads();
    for (int o = tid; o < HPC * kHeadDim; o += kThreads) {
        float A = 0.f;
        for (int g = 0; g < G; ++g) A += sm_acc[g * HPC * kHeadDim + o];
        const float L = s_L[o / kHeadDim];
        emit_out(a, seq, (size_t)h0 * kHeadDim + o, L > 0.f ? A / L : 0.f, pe);
    }
    step_done(a);
    DTRACE(4);
}

template <int HPC, int KT>
__global__ void __launch_bounds__(kThreads, 2) decode_kernel(DecodeArgs a) {
    decode_body<HPC, KT>(a);
}

template <int HPC, int KT>
cudaError_t launch_hpc(const DecodeArgs& a, cudaStream_t s) {
    static bool attr_set[64] = {};  // the attribute is per device
    const int smem = (int)decode_smem_bytes();
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(decode_kernel<HPC, KT>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) attr_set[dev] = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)a.total_splits, (unsigned)(a.n_kv * a.n_sub));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = (size_t)smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = a.pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, decode_kernel<HPC, KT>, a);
}

// The gather of a fused all-gather step: every element of the landing buffer of this step's
// parity, [world][rows][row_elems] tagged words, copied into dst [rows][world * row_elems] once
// its tag is this step's (bounded polling: a value that does not arrive records kErrWaitTimeout
// and the rest is skipped). The last CTA to finish advances the group's epoch. It lets its
// dependents launch at once: the next decode grid (a programmatic dependent) starts its prologue
// and first page copies meanwhile, and reads this grid's output only after its own wait.
__global__ void gather_ll_kernel(const unsigned long long* __restrict__ zone, unsigned long long* epoch,
                                 unsigned* done, int world, size_t slice, size_t rows, size_t row_elems,
                                 float* __restrict__ dst, int* err) {
    __shared__ unsigned long long s_e;
    grid_dep_launch();
    if (threadIdx.x == 0) s_e = *reinterpret_cast<volatile unsigned long long*>(epoch) + 1ull;
    __syncthreads();
    const unsigned long long e = s_e;
    const unsigned tag = (unsigned)e;
    const unsigned long long* base = zone + (size_t)(e & 1ull) * world * slice;
    const size_t rp = row_elems / 2, per_w = rows * rp, pairs = (size_t)world * per_w;
    long long budget = kWaitLimit;
    bool bad = false;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < pairs && !bad;
         i += (size_t)gridDim.x * blockDim.x) {
        const size_t w = i / per_w, rem = i % per_w, r = rem / rp, c = rem % rp;
        const unsigned long long* src = base + w * slice + r * row_elems + 2 * c;
        unsigned long long v0, v1;
        for (;;) {
            asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(v0), "=l"(v1) : "l"(src) : "memory");
            if ((unsigned)(v0 >> 32) == tag && (unsigned)(v1 >> 32) == tag) break;
            if (--budget <= 0) {
                bad = true;
                break;
            }
        }
        if (!bad)
            reinterpret_cast<float2*>(dst)[(r * world + w) * rp + c] =
                make_float2(__uint_as_float((unsigned)v0), __uint_as_float((unsigned)v1));
    }
    if (bad) *reinterpret_cast<volatile int*>(err) = kErrWaitTimeout;
    // launched as a programmatic dependent of the kernel that stores this rank's words (its
    // CTAs poll while that grid's tail runs): complete only after that grid has, so whatever
    // follows this kernel also follows it
    grid_dep_wait();
    __syncthreads();
    if (threadIdx.x == 0) {  // the step is over on this rank once every CTA is: the next may begin
        __threadfence();
        if (atomicAdd(done, 1u) == gridDim.x - 1) {
            *done = 0u;
            *reinterpret_cast<volatile unsigned long long*>(epoch) = e;
        }
    }
}

// Copies a host call's staged inputs (mapped pinned memory) into device memory. It lets its
// dependents launch at once, so the decode grid that follows (a programmatic dependent) runs its
// prologue and first page copies while the inputs cross the host link; that grid reads them
// only after griddepcontrol.wait.
__global__ void stage_copy_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst, size_t n16) {
    grid_dep_launch();
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += (size_t)gridDim.x * blockDim.x)
        dst[i] = src[i];
}

}  // namespace

cudaError_t launch_gather_ll(const unsigned long long* zone, unsigned long long* epoch, unsigned* done, int world,
                             size_t slice, size_t rows, size_t row_elems, float* dst, int* err, cudaStream_t s) {
    const size_t pairs = (size_t)world * rows * (row_elems / 2);
    // one 16-byte pair a thread while that fits in 4 CTAs an SM: every word is polled at once
    const unsigned blocks = (unsigned)std::max<size_t>(1, std::min<size_t>((pairs + 255) / 256, 148 * 4));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(blocks);
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, gather_ll_kernel, zone, epoch, done, world, slice, rows, row_elems, dst, err);
}

cudaError_t launch_stage_copy(void* dst, const void* src_mapped, size_t bytes, cudaStream_t s) {
    const size_t n16 = bytes / 16;
    if (!n16) return cudaSuccess;
    const unsigned blocks = (unsigned)std::min<size_t>(16, (n16 + 255) / 256);
    stage_copy_kernel<<<blocks, 256, 0, s>>>(static_cast<const uint4*>(src_mapped), static_cast<uint4*>(dst), n16);
    return cudaGetLastError();
}

// the ring, then one mbarrier per stage (fp8 rows: four times kStages stages)
size_t decode_smem_bytes() { return (size_t)kRingBytes + 4 * kStages * sizeof(uint64_t); }

template <int HPC>
cudaError_t launch_kt(const DecodeArgs& a, cudaStream_t s) {
    switch (a.pv.kind) {
        case kElemBF16: return launch_hpc<HPC, kElemBF16>(a, s);
        case kElemFP8: return launch_hpc<HPC, kElemFP8>(a, s);
        default: return launch_hpc<HPC, kElemF32>(a, s);
    }
}

cudaError_t launch_decode(const DecodeArgs& a, cudaStream_t s) {
    if (a.total_splits <= 0) return cudaSuccess;
    switch (a.hpc) {
        case 1: return launch_kt<1>(a, s);
        case 2: return launch_kt<2>(a, s);
        case 3: return launch_kt<3>(a, s);
        case 4: return launch_kt<4>(a, s);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace bebelm

#ifdef BEBELM_DECODE_TRACE
// timing build only: the last launch's per-CTA timeline (5 stamps per CTA, ns)
extern "C" __attribute__((visibility("default"))) int bebelm_debug_decode_trace(long long* out, int n_ctas) {
    return (int)cudaMemcpyFromSymbol(out, bebelm::g_dtrace, sizeof(long long) * 4 * 1024 * 8);
}
#endif
