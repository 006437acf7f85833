// Internal structures shared by the host runtime (api.cu) and the kernels.
// Not part of the public ABI (include/bebelm_attn.h is).
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_fp16.h>
#include <stddef.h>
#include <stdint.h>

namespace bebelm {

// Records `msg` as the calling thread's last error (bebelm_last_error) and returns code.
int set_last_error(int code, const char* msg);

constexpr int kHeadDim = 64;     // LFM2.5 head_dim (src/config.rs:20)
constexpr int kPageTokens = 64;  // positions per KV page
constexpr int kPageRowFloats = kPageTokens * kHeadDim;  // one kv head of one page: 4096 floats

// Device-side view of the page pool for one layer. A physical page p holds, for every
// layer l: K[l] then V[l], each a "block" [n_kv][64 tokens][64] of fp32, bf16 or fp8 (e4m3)
// elements.
// All offsets are in bytes.
struct PoolView {
    char* base;           // pool memory
    size_t page_bytes;    // one physical page (all layers, K and V)
    size_t layer_off;     // page start to this layer's K block
    size_t block_bytes;   // one K (or V) block = n_kv rows of a page
    int kind;             // element type: kElemF32, kElemBF16 or kElemFP8 (e4m3)
};

// A sequence's window for one layer: logical slots [base, base+len) live in
// logical pages slot/64, mapped through a ring table of `cap` entries.
struct SeqWindow {
    const int* table;
    int cap;
    int len;
    long long base;
};

// Bytes of one kv head of one page (64 tokens x 64 elements).
constexpr int kElemF32 = 0, kElemBF16 = 1, kElemFP8 = 2;
__host__ __device__ inline int elem_bytes(int kind) { return kind == kElemF32 ? 4 : kind == kElemBF16 ? 2 : 1; }
__host__ __device__ inline size_t row_bytes(const PoolView& pv) { return (size_t)kPageRowFloats * elem_bytes(pv.kind); }

// Byte offset of (slot, kv head, K or V) in the pool.
__host__ __device__ inline size_t slot_offset(const PoolView& pv, const int* table, int cap, long long slot, int kvh,
                                              int kind) {
    // logical pages stay below 2^32 (2^38 positions), so the ring index is a 32-bit modulo
    const unsigned lp = (unsigned)(slot >> 6);
    const int phys = table[lp % (unsigned)cap];
    return (size_t)phys * pv.page_bytes + pv.layer_off + (size_t)kind * pv.block_bytes + (size_t)kvh * row_bytes(pv) +
           (size_t)(slot & 63) * kHeadDim * elem_bytes(pv.kind);
}

#ifdef __CUDACC__
// Two e4m3 values (the low byte first) as floats; the conversion is exact.
__device__ __forceinline__ float2 fp8x2_to_float2(unsigned short v) {
    const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)v, __NV_E4M3);
    return __half22float2(*reinterpret_cast<const __half2*>(&h));
}
// Four e4m3 values packed in a word (element 0 in the low byte) as floats.
__device__ __forceinline__ float4 fp8x4_to_float4(uint32_t u) {
    const float2 a = fp8x2_to_float2((unsigned short)(u & 0xffffu)), b = fp8x2_to_float2((unsigned short)(u >> 16));
    return make_float4(a.x, a.y, b.x, b.y);
}
// x rounded to nearest e4m3 (saturating at +-448), returned as its byte.
__device__ __forceinline__ unsigned char float_to_fp8(float x) {
    return (unsigned char)__nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3);
}
// x as the cache of element type `kind` holds it.
__device__ __forceinline__ float round_to_kind(float x, int kind) {
    if (kind == kElemBF16) return __bfloat162float(__float2bfloat16_rn(x));
    if (kind == kElemFP8) return fp8x2_to_float2((unsigned short)float_to_fp8(x)).x;
    return x;
}
// Four consecutive elements (e..e+3) of the row at byte offset `off`, as floats.
__device__ __forceinline__ float4 kv_load4(const PoolView& pv, size_t off, int e) {
    if (pv.kind == kElemBF16) {
        const uint2 u = *reinterpret_cast<const uint2*>(pv.base + off + 2 * (size_t)e);
        return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u), __uint_as_float(u.y << 16),
                           __uint_as_float(u.y & 0xffff0000u));
    }
    if (pv.kind == kElemFP8) return fp8x4_to_float4(*reinterpret_cast<const uint32_t*>(pv.base + off + (size_t)e));
    return *reinterpret_cast<const float4*>(pv.base + off + 4 * (size_t)e);
}
// Stores four floats at elements e..e+3 (rounded to nearest-even bf16, or to nearest e4m3 with
// saturation, in a narrower pool).
__device__ __forceinline__ void kv_store4(const PoolView& pv, size_t off, int e, float4 v) {
    if (pv.kind == kElemBF16) {
        __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
        uint2 u;
        u.x = *reinterpret_cast<uint32_t*>(&a);
        u.y = *reinterpret_cast<uint32_t*>(&b);
        *reinterpret_cast<uint2*>(pv.base + off + 2 * (size_t)e) = u;
    } else if (pv.kind == kElemFP8) {
        const uint32_t u = (uint32_t)float_to_fp8(v.x) | ((uint32_t)float_to_fp8(v.y) << 8) |
                           ((uint32_t)float_to_fp8(v.z) << 16) | ((uint32_t)float_to_fp8(v.w) << 24);
        *reinterpret_cast<uint32_t*>(pv.base + off + (size_t)e) = u;
    } else {
        *reinterpret_cast<float4*>(pv.base + off + 4 * (size_t)e) = v;
    }
}
#endif

// ---- kernel 1: per-head RMSNorm + NEOX RoPE (+ KV append) ------------------
// Per-token destination when the tokens of one launch belong to different
// sequences (batched decode): token i goes to slot `slot` of `table` at `pos`.
struct AppendTarget {
    const int* table;
    int cap;
    long long slot;
    long long pos;
};

struct NormRopeArgs {
    // inputs, token-major: q [T][n_heads][hd], k/v [T][n_kv][hd] (k, v may be null)
    const float* q;
    const float* k;
    const float* v;
    const float* q_gain;
    const float* k_gain;
    int T, n_heads, n_kv, head_dim;
    long long pos0;
    float theta_scale;  // powf(theta, -2/head_dim), computed on the host like the reference
    float eps;
    int norm_q;         // 1: q heads are normed+roped; 0: q passes through
    int norm_k;         // 1: k heads are normed+roped; 0: k is appended raw
    // outputs
    float* q_out;            // [T][n_heads][hd] or null
    float* k_out;            // [T][n_kv][hd] contiguous or null
    __nv_bfloat16* q_bf16;   // optional bf16 copies [T][heads][64] for the prefill MMA
    __nv_bfloat16* k_bf16;
    __nv_bfloat16* v_bf16;
    // optional cache append (head_dim == 64 only)
    int append;
    PoolView pv;
    const int* table;
    int cap;
    long long slot0;  // logical slot of token 0
    const AppendTarget* targets;  // non-null: per-token table/slot/pos instead of the above
    int in_bf16;                  // q, k, v hold bf16 (head_dim 64 only)
    // input rows wider than this call's heads (a rank's heads of replicated full rows): a q row
    // holds q_row_heads heads of which this call's start at q_head0; likewise k/v (0: exactly
    // n_heads / n_kv, from 0)
    int q_row_heads, q_head0, kv_row_heads, kv_head0;
    // let the next kernel launch as a programmatic dependent at once (it must wait with
    // griddepcontrol.wait before reading anything this kernel writes: the tensor-core prefill)
    int trigger_dependents;
};
cudaError_t launch_norm_rope(const NormRopeArgs& a, cudaStream_t s);

// Copies a window [base, base+len) of one layer out of the pages, token-major
// [len][n_kv][64] (either output may be null).
cudaError_t launch_kv_gather(const PoolView& pv, const int* table, int cap, long long base, long long len,
                             int n_kv, float* k_out, float* v_out, cudaStream_t s);

// ---- kernel 3: split-K decode with fused combine (and fused norm/RoPE/append) --
struct DecodeSeq {
    const int* table;
    int cap;
    int len;            // window length, including a token appended by this launch
    long long base;     // first slot of the window
    int split0;         // first global split of this sequence
    int n_splits;       // splits of this sequence
    long long new_slot; // slot of the token this launch appends, or -1
    long long pos;      // RoPE position of that token (and of the query)
    long long dep_slot; // pages holding slots >= dep_slot are read only after griddepcontrol.wait
};

// Device-driven decode (step plans): step n of a plan appends slot slot0 + n at RoPE position
// pos0 + n and attends to the window that ends there (at most `window` positions). n lives
// in device memory; the last CTA of step n's grid advances it, so the launch arguments are
// the same for every step and the launch can be captured in a CUDA graph.
struct StepState {
    unsigned long long n;  // steps completed
    unsigned done;         // CTAs of the running step that have finished (reset by the last)
    unsigned pad;
};

struct DecodeArgs {
    const DecodeSeq* seqs;  // device array [n_seqs] (unused when n_seqs == 1)
    DecodeSeq one;          // the sequence itself when n_seqs == 1 (passed by value)
    int n_seqs;
    PoolView pv;
    // query: either already normed/roped (q) or raw (q_raw, normed+roped in-kernel)
    const float* q;         // [n_seqs][n_heads][64]
    const float* q_raw;     // [n_seqs][n_heads][64] or null
    // appended token (used when new_slot >= 0): raw k (normed+roped in-kernel) and v
    const float* k_new;     // [n_seqs][n_kv][64]
    const float* v_new;     // [n_seqs][n_kv][64]
    const float* q_gain;
    const float* k_gain;
    float theta_scale, eps;
    float* out;             // [n_seqs][n_heads][64]
    float* part_acc;        // [total_splits][n_kv*n_sub][hpc][64]
    float* part_ml;         // [total_splits][n_kv*n_sub][hpc][2]
    unsigned* counters;     // [n_seqs][n_kv*n_sub], zero between launches
    int* err;               // error word (device-visible; a timed-out wait stores its code)
    int n_heads, n_kv, group, hpc, n_sub;
    int pages_per_split;
    int total_splits;
    float scale_log2;       // score scale (1/sqrt(head_dim)) times log2(e)
    int pdl;                // launched as a programmatic dependent of the previous kernel
    // fused all-gather (KV-head sharding): when peer_world > 0 the final output of sequence 0
    // goes to every rank's landing zone instead of `out`, as tagged words (tag = the step's
    // epoch, see peer_epoch) at [(parity * peer_world + peer_rank) * n_heads*64 + head*64 + d]
    unsigned long long* const* peer_bufs;
    int peer_world, peer_rank;
    // device epoch word of the group: this step is *peer_epoch + 1
    const unsigned long long* peer_epoch;
    // step plan (one sequence): non-null step makes the window of `one` follow the counter
    StepState* step;
    long long step_slot0, step_pos0, step_len0, step_window;
    // the launch before this one was not this plan's: its previous step is at least two
    // launches back, hence complete when this grid starts (each decode grid triggers its
    // dependents only after its own griddepcontrol.wait), so the counter and every page may
    // be read before the wait
    int step_prewait;
    // the raw q/k/v and the gains were complete before the PDL predecessor passed its own wait
    // (they do not overlap the previous decode launch's output), so a CTA norms and ropes them
    // before griddepcontrol.wait; only the cache store of the new token waits
    int early_inputs;
    // test hook (bebelm_debug_expire_next_wait): CTA (0, 0) waits on a phase of its first stage
    // that nothing completes, with a short limit, so the launch takes the timeout path
    int expire_wait;
};
// Launches of the decode kernel still to be given expire_wait (set through the C-ABI for tests).
extern int g_expire_waits;
// The gather of a fused all-gather step (a landing zone of tagged words, see DecodeArgs): waits
// (bounded) for every element of this step's parity to carry this step's tag, copies them into
// dst [rows][world * row_elems], and advances *epoch (the last CTA; `done` counts them). It is
// launched as a programmatic dependent of the kernel before it (the one storing this rank's
// words): it polls during that grid's tail and completes only after that grid has.
cudaError_t launch_gather_ll(const unsigned long long* zone, unsigned long long* epoch, unsigned* done, int world,
                             size_t slice, size_t rows, size_t row_elems, float* dst, int* err, cudaStream_t s);
cudaError_t launch_decode(const DecodeArgs& a, cudaStream_t s);
// Copies `bytes` (a multiple of 16) from mapped pinned memory to device memory on s, letting
// the next kernel launch as a programmatic dependent right away.
cudaError_t launch_stage_copy(void* dst, const void* src_mapped, size_t bytes, cudaStream_t s);

size_t decode_smem_bytes();
constexpr int kDecodeMaxPagesPerSplit = 256;

// ---- kernel 2: causal prefill on the tensor cores ---------------------------
struct PrefillArgs {
    const __nv_bfloat16* q;  // [t][n_heads][64], normed + roped
    const __nv_bfloat16* k;  // [len_before + t][n_kv][64]: the window, oldest first
    const __nv_bfloat16* v;  // same
    float* out;              // [t][n_heads][64]
    int t, len_before, n_heads, n_kv;
    float scale_log2;        // score scale times log2(e)
    int* err;
    // fused all-gather (KV-head sharding): with peer_world > 0 the output rows go to every
    // rank's landing zone instead of `out`, as tagged words (see DecodeArgs):
    // [parity e&1][peer_rank][t][n_heads][64], e = *peer_epoch + 1, peer_slice words per rank
    unsigned long long* const* peer_bufs;
    const unsigned long long* peer_epoch;
    int peer_world, peer_rank;
    size_t peer_slice;
};
// TMA descriptors of q, k, v (opaque 128-byte CUtensorMap objects).
struct alignas(64) PrefillMaps {
    unsigned char q[128], k[128], v[128];
};
bool prefill_make_maps(const PrefillArgs& a, PrefillMaps* m);  // host only; false on failure
cudaError_t launch_prefill(const PrefillArgs& a, const PrefillMaps& m, cudaStream_t s);
// Window [base, base+len) of one layer as bf16, token-major [len][n_kv][64].
cudaError_t launch_kv_gather_bf16(const PoolView& pv, const int* table, int cap, long long base, long long len,
                                  int n_kv, __nv_bfloat16* k_out, __nv_bfloat16* v_out, cudaStream_t s);

// device error codes written to DecodeArgs::err
constexpr int kErrWaitTimeout = 1;

// GGML weight types of the quantized products (ggml's type ids, src/tensor.rs:41-62)
constexpr int kGgmlF32 = 0, kGgmlF16 = 1, kGgmlQ4K = 12, kGgmlQ6K = 14;
size_t ggml_row_bytes(int dtype, size_t n_in);  // 0 for an unsupported dtype
// activations [n_tokens][n_in] (n_in a multiple of 256) -> int8 quants, per-256 scales,
// per-32 sums, in token-major order
cudaError_t launch_quantize_q8(const float* x, size_t n_in, size_t n_tokens, int8_t* q, float* scales, int* sums,
                               cudaStream_t s);
// y [n_tokens][n_out] = W x; K-quant weights take the Q8 activations, F32/F16 weights x itself
cudaError_t launch_qmatmul(int dtype, const uint8_t* w, size_t n_in, size_t n_out, const float* x, size_t n_tokens,
                           const int8_t* q8, const float* q8_scales, const int* q8_sums, float* y, int* err,
                           cudaStream_t s);
// Q4_K / Q6_K weights, many tokens, on the tensor cores (tcgen05 kind::i8); same bits as
// launch_qmatmul. A bounded wait that gives up stores kErrWaitTimeout to *err.
// cudaErrorNotSupported (nothing launched) when the buffers cannot be described to TMA.
cudaError_t launch_kquant_tc(int dtype, const uint8_t* w, size_t n_in, size_t n_out, size_t n_tokens,
                             const int8_t* q8, const float* q8_scales, const int* q8_sums, float* y, int* err,
                             cudaStream_t s);
// whether launch_qmatmul sends K-quant batches to launch_kquant_tc (on unless BEBELM_QMM_TC=0)
bool kquant_tc_enabled();
cudaError_t launch_dequantize(int dtype, const uint8_t* data, size_t n, float* out, cudaStream_t s);
// one token, up to 3 matrices sharing the input x [n_in <= 8192]: y_i = W_i x, x quantized
// to Q8 inside the kernel (K-quant segments); results identical to launch_qmatmul
struct QmvSegs {
    int n;
    int dtype[3];
    const uint8_t* w[3];
    size_t row_bytes[3], n_out[3];
    float* y[3];
};
cudaError_t launch_qmv_multi(const QmvSegs& segs, const float* x, size_t n_in, cudaStream_t s);
// one token against a large K-quant matrix (rows streamed by bulk copies; same bits as
// launch_qmv_multi). cudaErrorNotSupported (nothing launched) for other dtypes, row sizes that
// are not 16-byte multiples or unaligned weights. A wait that gives up stores to *err.
cudaError_t launch_qmv_stream(int dtype, const uint8_t* w, size_t n_out, const float* x, size_t n_in, float* y,
                              int* err, cudaStream_t s);
// the logits head in one launch (same bits as launch_rmsnorm_row + launch_qmv_multi +
// launch_greedy): logits [vocab] = W rmsnorm(h, gain, eps), *token = argmax (nullable).
// cand_v / cand_i: one slot per SM; *counter: 0 between calls (re-armed by the kernel).
cudaError_t launch_head_stream(int dtype, const uint8_t* w, size_t vocab, const float* h, const float* gain, float eps,
                               size_t hidden, float* logits, uint32_t* token, float* cand_v, uint32_t* cand_i,
                               unsigned* counter, int* err, cudaStream_t s);

// logits head (head.cu): final RMSNorm of one hidden state [n <= 8192], one CTA
cudaError_t launch_rmsnorm_row(const float* x, const float* gain, int n, float eps, float* out, cudaStream_t s);
// Sampler::sample with temperature <= 0: presence penalty (when penalty != 1 and history is
// non-empty; bitmap = (n + 31) / 32 words of scratch) on logits in place, then argmax -> *token
cudaError_t launch_greedy(float* logits, size_t n, const uint32_t* history, size_t n_history, float penalty,
                          uint32_t* bitmap, uint32_t* token, cudaStream_t s);


}  // namespace bebelm
