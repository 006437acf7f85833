/*
 * bebelm_attn.h — C-ABI of the B200 (sm_100a) attention library for BebeLM.
 *
 * Replaces the grouped-query attention hot path of the reference Rust crate
 * (maximecb/bebelm 0.3.6): the per-head q/k RMSNorm + NEOX RoPE, the KV-cache
 * append, single-query decode attention, the per-token causal prefill loop, and
 * the host `Cache` type those read. Each entry point names the reference
 * interface it stands in for.
 *
 * Conventions
 *  - Every function returns int: 0 on success, a negative BEBELM_ERR_* code on
 *    failure; bebelm_last_error() returns the message of the calling thread's
 *    last failure. No C++ exception crosses this boundary.
 *  - `mem` says where the float buffers of a call live: BEBELM_MEM_HOST (any
 *    host memory; the call copies through pinned staging and synchronises the
 *    stream before returning) or BEBELM_MEM_DEVICE (device pointers on the
 *    handle's GPU; the call only enqueues work on `stream`).
 *  - `stream` is a cudaStream_t passed as void*; NULL means the legacy default
 *    stream of the current thread.
 *  - Handles are opaque. Calls on one handle (or on sequences of one pool) are
 *    not thread-safe and must be ordered on one stream: they share the pool's
 *    scratch memory.
 *  - Geometry: head_dim <= 64 for the drop-ins (padded to 64 internally);
 *    caches and fused calls take head_dim == 64 and page_tokens == 64.
 *    n_heads must be a multiple of n_kv_heads (GQA group = n_heads/n_kv_heads).
 */
#ifndef BEBELM_ATTN_H
#define BEBELM_ATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define BEBELM_API __attribute__((visibility("default")))
#else
#define BEBELM_API
#endif

#define BEBELM_ABI_VERSION 1

enum {
    BEBELM_OK = 0,
    BEBELM_ERR_INVALID = -1,     /* bad argument, geometry or handle */
    BEBELM_ERR_CUDA = -2,        /* a CUDA runtime call failed */
    BEBELM_ERR_OOM = -3,         /* device or pinned allocation failed */
    BEBELM_ERR_CAPACITY = -4,    /* the window would exceed the cache's capacity */
    BEBELM_ERR_UNSUPPORTED = -5, /* geometry/dtype this build does not implement */
    BEBELM_ERR_TIMEOUT = -7,     /* a bounded device-side wait gave up */
    BEBELM_ERR_NO_DEVICE = -8,   /* no CUDA device, or the device is not sm_100 */
    BEBELM_ERR_FORMAT = -9,      /* malformed GGUF file, or metadata that does not match the model */
    BEBELM_ERR_NOT_FOUND = -10,  /* no such GGUF tensor or metadata key (of the asked type) */
    BEBELM_ERR_IO = -11          /* a file could not be opened, read or mapped */
};

enum { BEBELM_MEM_HOST = 0, BEBELM_MEM_DEVICE = 1 };
enum { BEBELM_F32 = 0, BEBELM_BF16 = 1 };
/* cache dtype only: K and V stored as fp8 e4m3 (one byte each) */
enum { BEBELM_FP8_E4M3 = 3 };
/* bebelm_attn_prefill only: fp32 inputs (as the reference's attn_batch passes them), attention
 * on the tensor cores. */
enum { BEBELM_F32_TENSOR = 2 };

typedef struct bebelm_kv_pool bebelm_kv_pool; /* device page pool + scratch */
typedef struct bebelm_kv bebelm_kv;           /* one sequence's KV window */

/* ---------------------------------------------------------------- misc --- */
BEBELM_API int bebelm_abi_version(void);
/* Copies the calling thread's last error message (NUL-terminated, truncated to n). */
BEBELM_API int bebelm_last_error(char* buf, size_t n);
/* Number of visible sm_100 devices. */
BEBELM_API int bebelm_device_count(int* n);

/* ------------------------------------------------------------ drop-ins --- */
/* Replaces `attention_decode(q, k, v, n_ctx, n_heads, n_kv_heads, head_dim, out)`
 * (src/kernels/attention.rs:17-26). Host buffers: q/out [n_heads*head_dim],
 * k/v token-major [n_ctx][n_kv_heads][head_dim]. Copies K/V to the current
 * device each call, so it serves parity tests and one-off calls; the
 * cache-resident path is bebelm_attn_step. n_ctx == 0 writes zeros. */
BEBELM_API int bebelm_attn_decode_host(const float* q, const float* k, const float* v, size_t n_ctx,
                            int n_heads, int n_kv_heads, int head_dim, float* out);

/* Replaces `norm_rope_heads(buf, n_heads, gain, pos)` (src/model.rs:600-608),
 * i.e. `rmsnorm` (src/kernels/rmsnorm.rs:10-21) then `rope_neox`
 * (src/kernels/rope.rs:16-29) per head, in place, for n_tokens consecutive
 * positions pos0, pos0+1, ... buf is [n_tokens][n_heads][head_dim]. head_dim
 * even and <= 64. The reference fixes theta = 5e6 and eps = 1e-5
 * (src/config.rs:31-32); both are arguments here. */
BEBELM_API int bebelm_norm_rope_heads(float* buf, size_t n_tokens, int n_heads, int head_dim,
                           const float* gain, size_t pos0, float theta, float eps, int mem,
                           void* stream);

/* ------------------------------------------------------------- KV cache --- */
/* Device replacement for `Cache` (src/cache.rs:9-49), attention layers only.
 * Storage is paged: a page holds `page_tokens` (64) positions of K and V for
 * every attention layer, laid out [layer][K|V][kv_head][token][64]. dtype
 * BEBELM_F32 keeps the reference's fp32 history; BEBELM_BF16 stores K and V
 * rounded to bf16 (nearest even) when appended, halving the bytes each decode
 * step reads, with attention still computed in fp32. BEBELM_FP8_E4M3 stores them
 * as e4m3 (nearest, saturating at +-448): a quarter of the fp32 bytes; e4m3 keeps
 * 3 mantissa bits, so each stored value carries up to 2^-4 relative rounding
 * (the reference's planned reduced-precision cache, design.md:451).
 * A sequence's window is a ring of pages, so evict_front (the sliding window
 * of src/agent.rs:471-476) moves an offset and recycles whole pages instead of
 * moving memory. The ring has ceil(max_context/64) + 2 pages: a window always
 * fits max_context + page_tokens positions per layer (a page more when it
 * starts on a page boundary); an append beyond the ring fails with
 * BEBELM_ERR_CAPACITY and changes nothing. */
BEBELM_API int bebelm_kv_pool_create(int n_layers, int n_kv_heads, int head_dim, size_t n_pages,
                          int page_tokens, int dtype, int device, bebelm_kv_pool** out);
BEBELM_API int bebelm_kv_pool_destroy(bebelm_kv_pool* pool);
BEBELM_API int bebelm_kv_pool_free_pages(const bebelm_kv_pool* pool, size_t* out);

/* `Cache::new()` (src/cache.rs:22-29): a sequence with its own private pool. */
BEBELM_API int bebelm_kv_create(int n_layers, int n_kv_heads, int head_dim, size_t max_context,
                     int page_tokens, int dtype, int device, bebelm_kv** out);
/* A sequence drawing pages from a shared pool (batched decode requires this). */
BEBELM_API int bebelm_kv_create_in_pool(bebelm_kv_pool* pool, size_t max_context, bebelm_kv** out);
BEBELM_API int bebelm_kv_destroy(bebelm_kv* kv);
/* `#[derive(Clone)]` on Cache (src/cache.rs:9; Agent fork, src/agent.rs:92):
 * a deep copy. A private-pool sequence clones into a new private pool; a
 * shared-pool sequence clones into new pages of the same pool. */
BEBELM_API int bebelm_kv_clone(const bebelm_kv* src, bebelm_kv** dst);
/* `Agent::clear` replacing the cache with `Cache::new()` (src/agent.rs:479-483). */
BEBELM_API int bebelm_kv_clear(bebelm_kv* kv);
/* `Cache::kv_len` (src/cache.rs:33-35): longest layer window, in positions. */
BEBELM_API int bebelm_kv_len(const bebelm_kv* kv, size_t* out);
BEBELM_API int bebelm_kv_layer_len(const bebelm_kv* kv, int layer, size_t* out);
/* `Cache::pos` (src/cache.rs:18): the next token's absolute position. */
BEBELM_API int bebelm_kv_pos(const bebelm_kv* kv, size_t* out);
BEBELM_API int bebelm_kv_set_pos(bebelm_kv* kv, size_t pos);
/* `Cache::evict_front(n)` (src/cache.rs:40-48): drop the oldest n positions of
 * every layer holding at least n; pos is not rewound. */
BEBELM_API int bebelm_kv_evict_front(bebelm_kv* kv, size_t n);
/* `cache.k[layer].extend_from_slice(k)` + same for v (src/model.rs:443-444,
 * 241-242): append t positions of already-normed/roped k and raw v,
 * token-major [t][n_kv_heads][head_dim]. */
BEBELM_API int bebelm_kv_append(bebelm_kv* kv, int layer, const float* k, const float* v, size_t t,
                     int mem, void* stream);
/* Reads layer's window back token-major [len][n_kv_heads][head_dim] (what
 * `cache.k[layer]` / `cache.v[layer]` hold in the reference). Either pointer
 * may be NULL. */
BEBELM_API int bebelm_kv_read(const bebelm_kv* kv, int layer, float* k_out, float* v_out, int mem,
                   void* stream);

/* ----------------------------------------------------------- fused ops --- */
/* The middle of `attn_step` (src/model.rs:440-451): q/k norm + RoPE at `pos`,
 * append k and v to layer's window, single-query GQA attention over the whole
 * window. q [n_heads*64], k/v [n_kv_heads*64], gains [64], out [n_heads*64].
 * q is not modified (the reference's in-place q is an internal temporary). */
BEBELM_API int bebelm_attn_step(bebelm_kv* kv, int layer, int n_heads, const float* q, const float* k,
                     const float* v, const float* q_gain, const float* k_gain, float theta,
                     float eps, size_t pos, float* out, int mem, void* stream);

/* `attention_decode` (src/kernels/attention.rs:17-55) over layer's cached
 * window without appending: q [n_heads*64] already normed and roped (as the
 * reference's q is when it reaches attention_decode), out [n_heads*64]. This is
 * the call a Rust `attention_decode` shim makes once K/V live on the device. */
BEBELM_API int bebelm_attn_decode_cached(const bebelm_kv* kv, int layer, int n_heads, const float* q, float* out,
                                         int mem, void* stream);

/* No counterpart in the reference. bebelm_attn_decode_cached, but allocating
 * nothing: for callers that cannot call cudaMalloc while they decode — e.g. a
 * host whose device memory is fully reserved by another allocator, or a token
 * loop that must not take the device-wide synchronisation cudaMalloc can cause.
 * The split scratch is a fixed 2 MiB device array inside this library (held by
 * every GPU that loads it, until exit) instead of the pool's on-demand scratch.
 * Device pointers only (q normed and roped, [n_heads*64]; out [n_heads*64]).
 * The first call on a device looks up the array's address and clears its
 * counters (do that call before any stream capture). A window too large for
 * the array is rejected with BEBELM_ERR_INVALID. All calls share the array:
 * calls that overlap on the GPU (different streams, or another thread) race.
 * A bounded device-side wait that gives up is recorded in kv's pool error word,
 * like every other call on the pool: bebelm_kv_check reports it and then also
 * clears the array's split counters, so the next call starts clean. */
BEBELM_API int bebelm_attn_decode_cached_noalloc(const bebelm_kv* kv, int layer, int n_heads, const float* q,
                                                 float* out, void* stream);

/* The middle of `attn_batch` (src/model.rs:232-254): t tokens at positions
 * pos0.. are normed/roped, appended, and each attends causally to the window
 * up to and including itself. q [t][n_heads*64], k/v [t][n_kv_heads*64] in
 * `in_dtype` (BEBELM_F32 or BEBELM_BF16); out [t][n_heads*64] fp32. The cache
 * always stores the fp32 normed/roped k and raw v. BEBELM_BF16 inputs run the
 * attention on the tensor cores (tcgen05, bf16 operands, fp32 accumulation,
 * within 2e-2 relative of the reference); BEBELM_F32 inputs keep the reference's
 * fp32 arithmetic on the CUDA cores (within 1e-3 absolute). BEBELM_F32_TENSOR takes
 * fp32 inputs like BEBELM_F32, norms and ropes them in fp32 (the cache gets the
 * same fp32 k as with BEBELM_F32) and rounds the normed q, k and the v to bf16 for
 * the tensor-core attention: the BEBELM_BF16 speed for an fp32 caller, within the
 * same 2e-2 relative. */
BEBELM_API int bebelm_attn_prefill(bebelm_kv* kv, int layer, int n_heads, const void* q, const void* k,
                        const void* v, int in_dtype, size_t t, size_t pos0,
                        const float* q_gain, const float* k_gain, float theta, float eps,
                        float* out, int mem, void* stream);

/* Batched decode across independent sequences (one Agent each) that share one
 * pool: for sequence i, the attn_step of its token at pos[i]. q [n][n_heads*64],
 * k/v [n][n_kv_heads*64], out [n][n_heads*64]; pos is a host array. */
BEBELM_API int bebelm_attn_decode_batched(bebelm_kv* const* seqs, int n_seqs, int layer, int n_heads,
                               const float* q, const float* k, const float* v,
                               const float* q_gain, const float* k_gain, float theta, float eps,
                               const size_t* pos, float* out, int mem, void* stream);

/* Synchronises `stream` and reports whether a bounded device-side wait of any
 * call on kv's pool gave up since the last check (BEBELM_ERR_TIMEOUT; the flag
 * is then cleared). Host-memory calls check this themselves; device-memory
 * calls only enqueue work, so their callers check here. */
BEBELM_API int bebelm_kv_check(const bebelm_kv* kv, void* stream);

/* Testing only; no counterpart in the reference. Makes the next `n_launches`
 * decode-kernel launches (any entry point that decodes) take their timeout path:
 * the first CTA first waits, with a short limit, on a barrier nothing completes,
 * records BEBELM_ERR_TIMEOUT in the pool's error word and leaves once its own
 * copies have landed. No GPU fault is involved. Lets a test check that a wait
 * that gives up is reported and that the next call is correct again. */
BEBELM_API int bebelm_debug_expire_next_wait(int n_launches);

/* ---------------------------------------------- quantized weights (GGML) --- */
/* The projections that feed the path (src/model.rs:434-436, 454) multiply GGML-quantized
 * weights by f32 activations. Weight dtypes are ggml's type ids. W is [n_out rows][n_in],
 * each row packed in the dtype's blocks (row-major by output, as stored in the GGUF). */
enum { BEBELM_GGML_F32 = 0, BEBELM_GGML_F16 = 1, BEBELM_GGML_Q4_K = 12, BEBELM_GGML_Q6_K = 14 };
/* `matvec(dtype, w, n_in, n_out, x, y)` (src/kernels/matmul.rs:850-905): y[n_out] = W x.
 * Q4_K/Q6_K weights take the reference's Q8-activation integer dot (quantize_q8 of x per
 * 256-block, exact i32 block dots, f32 block scaling, blocks summed in order): bit for bit
 * the reference's result. F32/F16 weights use the reference's `dot` structure (its final
 * 8-lane reduction order is not visible; within f32 rounding of the reference). n_in must be
 * a multiple of 256 for K-quants. */
BEBELM_API int bebelm_matvec(int dtype, const void* w, size_t n_in, size_t n_out, const float* x, float* y,
                             int mem, void* stream);
/* `matmul(..., n_tokens, y)` (src/kernels/matmul.rs:908-1013): token-major x [n_tokens][n_in],
 * y [n_tokens][n_out]; bit-identical to matvec per token, as the reference's is. */
BEBELM_API int bebelm_matmul(int dtype, const void* w, size_t n_in, size_t n_out, const float* x,
                             size_t n_tokens, float* y, int mem, void* stream);
/* `dequantize_into(dtype, data, out)` (src/kernels/dequant.rs:151-176): n_elements f32. */
BEBELM_API int bebelm_dequantize(int dtype, const void* data, size_t n_elements, float* out, int mem,
                                 void* stream);

/* The whole attention operator of a layer on device-resident weights. The weights are the
 * layer's GGUF tensors as stored (attn_q [n_heads*64][hidden], attn_k / attn_v
 * [n_kv*64][hidden], attn_output [hidden][n_heads*64], each a GGML dtype above) plus the
 * q/k norm gains [64]; create copies them to `device` once (host pointers). */
typedef struct bebelm_attn_weights bebelm_attn_weights;
BEBELM_API int bebelm_attn_weights_create(int device, int n_heads, int n_kv_heads, size_t hidden,
                                          int dtype_q, const void* wq, int dtype_k, const void* wk,
                                          int dtype_v, const void* wv, int dtype_o, const void* wo,
                                          const float* q_gain, const float* k_gain,
                                          bebelm_attn_weights** out);
BEBELM_API int bebelm_attn_weights_destroy(bebelm_attn_weights* w);
/* `attn_step(layer, x, pos, cache)` (src/model.rs:430-455) whole: q/k/v = W x (matvec),
 * norm + RoPE, append, attention over the window, out = W_o attn. x, out [hidden]. */
BEBELM_API int bebelm_attn_layer_step(bebelm_kv* kv, int layer, const bebelm_attn_weights* w,
                                      const float* x, size_t pos, float theta, float eps, float* out,
                                      int mem, void* stream);
/* `attn_batch(layer, x, pos0, t, cache)` (src/model.rs:224-258) whole: the projections over
 * t tokens (matmul), then the causal prefill of the chunk, then W_o. x, out [t][hidden].
 * tensor_cores 1: attention on the tensor cores (bf16 operands, within 2e-2 relative);
 * 0: the reference's fp32 arithmetic (within 1e-3). */
BEBELM_API int bebelm_attn_layer_batch(bebelm_kv* kv, int layer, const bebelm_attn_weights* w,
                                       const float* x, size_t t, size_t pos0, int tensor_cores,
                                       float theta, float eps, float* out, int mem, void* stream);

/* ---------------------------------------------------- step plans (graphs) --- */
/* No counterpart in the reference. Device-driven decode steps, for a token loop captured
 * once in a CUDA graph and replayed: the host work of bebelm_attn_step (slot bookkeeping,
 * split plan, page assignment) is done once when the plan is created, and the kernel keeps
 * the window state itself. Step n of a plan (n = 0, 1, ... counted on the device) is the
 * attn_step of a token at RoPE position pos + n, where pos is the cache's pos when the plan
 * was created (bebelm_kv_set_pos): its k/v are appended after the layer's window and it
 * attends to the last min(len + n + 1, window) positions (len = the layer's window length at
 * creation), i.e. the window slides by one position per step once full, as the Agent's
 * trim_context does (src/agent.rs:466-476). window 0 means max_context.
 *  - create: gives every entry of the sequence's page ring a physical page (so no step needs
 *    the host), and fails if another non-empty layer's window differs from this layer's
 *    (the model steps all layers in lockstep: one plan per layer, each launched per token).
 *  - launch: device pointers only (q [n_heads*64], k/v [n_kv_heads*64], gains [64], out
 *    [n_heads*64]); allocates, copies and synchronises nothing, so it may be captured. Each
 *    launch is one step; steps of one plan must run in stream order.
 *  - steps: synchronises the stream and reports the steps taken so far.
 *  - finish: synchronises, folds the steps into the cache (window, pos) and frees the plan.
 * While a cache has open plans, every other call on it fails with BEBELM_ERR_INVALID. */
typedef struct bebelm_step_plan bebelm_step_plan;
BEBELM_API int bebelm_step_plan_create(bebelm_kv* kv, int layer, int n_heads, size_t window,
                                       bebelm_step_plan** out);
BEBELM_API int bebelm_step_plan_launch(bebelm_step_plan* plan, const float* q, const float* k,
                                       const float* v, const float* q_gain, const float* k_gain,
                                       float theta, float eps, float* out, void* stream);
BEBELM_API int bebelm_step_plan_steps(const bebelm_step_plan* plan, unsigned long long* n, void* stream);
BEBELM_API int bebelm_step_plan_finish(bebelm_step_plan* plan, void* stream);
/* The same for the whole attention operator (bebelm_attn_layer_step): a plan made with the
 * layer's uploaded weights also owns the scratch of its projections, and each
 * bebelm_step_plan_launch_layer is one token: x [hidden] -> out [hidden], device pointers.
 * It enqueues the Q8 quantization of x, the q/k/v projections, the plan's decode step, the Q8
 * quantization of the attention output and the output projection; none of them allocates,
 * copies or synchronises. steps/finish as above. */
BEBELM_API int bebelm_step_plan_create_layer(bebelm_kv* kv, int layer, const bebelm_attn_weights* w,
                                             size_t window, bebelm_step_plan** out);
BEBELM_API int bebelm_step_plan_launch_layer(bebelm_step_plan* plan, const float* x, float theta,
                                             float eps, float* out, void* stream);

/* ------------------------------------------- multi-GPU (KV-head sharding) --- */
/* Fused decode + all-gather for KV-head sharding over NVLink, one process per
 * GPU. The reference runs every head on one CPU (src/model.rs:440-451); here
 * rank r of `world` holds kv heads [r*n_kv, (r+1)*n_kv) of the model and their
 * query heads, and the full [world * n_heads * 64] output of the step lands
 * on every rank without a separate collective: the kernel's output-writing
 * CTAs store their heads straight into every rank's landing zone (peer
 * stores over NVLink), each value in an 8-byte word tagged with the step's
 * number; a one-block kernel then polls its own zone (bounded) until every
 * word carries this step's tag and copies the values out. No fence or flag
 * sits between the stores and the reader.
 *
 * Setup is collective: every rank calls bebelm_peer_group_create (which
 * allocates its zone and writes a BEBELM_IPC_HANDLE_BYTES handle), the caller
 * exchanges the handles (e.g. an all_gather over torch.distributed), then every
 * rank calls bebelm_peer_group_connect with all `world` handles in rank order.
 * slice_floats is one rank's output, n_heads*64. Steps must be called by all
 * ranks in the same order with the same geometry and window lengths; a rank
 * that stops calling makes its peers' next step fail with BEBELM_ERR_TIMEOUT
 * (seen by bebelm_kv_check, or at once for host-memory calls). Destroy is
 * collective too: barrier on the host after the last step, then destroy. */
#define BEBELM_IPC_HANDLE_BYTES 64
typedef struct bebelm_peer_group bebelm_peer_group;
BEBELM_API int bebelm_peer_group_create(int device, int world, int rank, size_t slice_floats,
                                        void* handle_out, bebelm_peer_group** out);
BEBELM_API int bebelm_peer_group_connect(bebelm_peer_group* g, const void* handles);
BEBELM_API int bebelm_peer_group_destroy(bebelm_peer_group* g);
/* bebelm_attn_step on this rank's heads, gathered: q [n_heads*64] and k/v
 * [n_kv_heads*64] are this rank's slices, out [world*n_heads*64] is the full
 * output in rank (= head) order. */
BEBELM_API int bebelm_attn_step_allgather(bebelm_kv* kv, bebelm_peer_group* g, int layer, int n_heads,
                                          const float* q, const float* k, const float* v,
                                          const float* q_gain, const float* k_gain, float theta,
                                          float eps, size_t pos, float* out, int mem, void* stream);
/* bebelm_attn_prefill on this rank's heads, gathered (device memory): q [t][world*n_heads*64]
 * and k/v [t][world*n_kv_heads*64] are the full, replicated input rows (the call takes its
 * rank's heads from them); out [t][world*n_heads*64] receives every rank's heads. The
 * tensor-core prefill stores its output rows straight into every rank's landing zone (NVLink
 * stores of tagged words from the kernel's epilogue); a gather kernel polls the tags and
 * copies the rows into `out`. in_dtype BEBELM_BF16 or BEBELM_F32_TENSOR. The group's slice_floats must hold
 * t*n_heads*64 (BEBELM_ERR_CAPACITY otherwise): make a separate group for prefill, sized for
 * the largest chunk. */
BEBELM_API int bebelm_attn_prefill_allgather(bebelm_kv* kv, bebelm_peer_group* g, int layer, int n_heads,
                                             const void* q, const void* k, const void* v, int in_dtype, size_t t,
                                             size_t pos0, const float* q_gain, const float* k_gain, float theta,
                                             float eps, float* out, void* stream);
/* A step plan's step (bebelm_step_plan_launch, device memory) on this rank's heads, gathered
 * the same way: out [world*n_heads*64]. The group counts its steps in device memory (the
 * epoch that picks the landing buffer and tags the words), so a CUDA graph of
 * these steps, captured once on every rank, replays with no host work. Every rank's plans
 * must step in the same order, and replays must be launched on all ranks. */
BEBELM_API int bebelm_step_plan_launch_allgather(bebelm_step_plan* plan, bebelm_peer_group* g,
                                                 const float* q, const float* k, const float* v,
                                                 const float* q_gain, const float* k_gain, float theta,
                                                 float eps, float* out, void* stream);

/* ---- logits head and greedy token choice (next after the projections) ----
 * Replaces Model::logits_from_hidden (src/model.rs:379-388: final RMSNorm with
 * token_embd_norm, then the tied token_embd matvec) and, for temperature <= 0,
 * Sampler::sample (src/sampler.rs:64-88) with argmax (src/sampler.rs:139-149).
 * token_embd is uploaded once as stored (ggml dtype, [vocab][hidden], hidden <= 8192). */
typedef struct bebelm_head bebelm_head;
BEBELM_API int bebelm_head_create(int device, int dtype, const void* token_embd, size_t hidden, size_t vocab,
                                  const float* norm_gain, bebelm_head** out);
BEBELM_API int bebelm_head_destroy(bebelm_head* head);
/* h [hidden] -> logits [vocab] (nullable) and the greedy token (argmax, nullable). Device
 * memory: with logits null the head's own buffer holds them; nothing leaves the device. */
BEBELM_API int bebelm_head_logits(bebelm_head* head, const float* h, float eps, float* logits,
                                  uint32_t* token, int mem, void* stream);
/* Sampler::sample with temperature <= 0: when repeat_penalty != 1, each distinct token of
 * history [n_history] once: l > 0 ? l / p : l * p (logits rewritten in place, as the
 * reference does); then the first index of the maximum (NaN never wins; 0 when no logit
 * is above -inf). Host history ids must be < n (BEBELM_ERR_INVALID otherwise); device
 * history ids >= n are ignored. */
BEBELM_API int bebelm_sample_greedy(float* logits, size_t n, const uint32_t* history, size_t n_history,
                                    float repeat_penalty, uint32_t* token, int mem, void* stream);

/* ------------------------------------------------------------- GGUF weights ---
 * The reference's GGUF reader (src/gguf.rs): GgufFile::open memory-maps a file and
 * GgufFile::from_bytes parses a buffer (here: a copy of it); both parse the header,
 * the metadata key/values and the tensor table, and check that each tensor's bytes lie
 * inside the file. Failures return BEBELM_ERR_FORMAT with the reference's GgufError
 * wording (bad magic, unsupported version, unexpected end of file, unknown metadata
 * value type, invalid UTF-8, unmodeled ggml type, data range outside the file), or
 * BEBELM_ERR_IO. A handle is immutable after parsing: it may be read from any thread.
 * Pointers it hands out (names, strings, tensor data) live until bebelm_gguf_close. */
typedef struct bebelm_gguf bebelm_gguf;
#define BEBELM_GGUF_MAX_DIMS 8
/* TensorInfo (src/gguf.rs:120-139). dims fastest-varying first; offset is relative to
 * the data section, data_start absolute in the file; data points at the bytes. */
typedef struct {
    const char* name;
    size_t name_len; /* bytes of name (a name may hold a NUL byte) */
    uint32_t n_dims; /* may exceed BEBELM_GGUF_MAX_DIMS; only the first ones are in dims */
    uint64_t dims[BEBELM_GGUF_MAX_DIMS];
    uint64_t n_elements;
    int ggml_type;
    uint64_t offset, data_start, data_len;
    const void* data;
} bebelm_gguf_tensor;
BEBELM_API int bebelm_gguf_open(const char* path, bebelm_gguf** out);
BEBELM_API int bebelm_gguf_from_bytes(const void* data, size_t n, bebelm_gguf** out);
BEBELM_API int bebelm_gguf_close(bebelm_gguf* g);
/* GgufFile's version, alignment (general.alignment, default 32), data_offset, and counts. */
BEBELM_API int bebelm_gguf_header(const bebelm_gguf* g, uint32_t* version, uint64_t* alignment,
                                  uint64_t* data_offset, size_t* n_tensors, size_t* n_kv);
/* GgufFile::tensors[i], and Model::tensor by name (src/model.rs:79-81; BEBELM_ERR_NOT_FOUND). */
BEBELM_API int bebelm_gguf_tensor_at(const bebelm_gguf* g, size_t i, bebelm_gguf_tensor* out);
BEBELM_API int bebelm_gguf_find_tensor(const bebelm_gguf* g, const char* name, bebelm_gguf_tensor* out);
/* The i-th distinct metadata key in file order, its byte length (a key may hold a NUL byte;
 * the lookups below take NUL-terminated keys) and its value type (the GGUF discriminant). */
BEBELM_API int bebelm_gguf_key_at(const bebelm_gguf* g, size_t i, const char** key, size_t* key_len,
                                  int* value_type);
/* The typed accessors of src/gguf.rs:196-283: get_u32 widens any integer type, get_f32
 * takes F32 or F64, get_u32_array any integer array (copies up to cap, *len = its length),
 * get_str copies up to cap-1 bytes and a NUL (*len = its byte length). A missing key or
 * another type gives BEBELM_ERR_NOT_FOUND, as the reference's None. */
BEBELM_API int bebelm_gguf_get_u32(const bebelm_gguf* g, const char* key, uint32_t* out);
BEBELM_API int bebelm_gguf_get_f32(const bebelm_gguf* g, const char* key, float* out);
BEBELM_API int bebelm_gguf_get_str(const bebelm_gguf* g, const char* key, char* buf, size_t cap, size_t* len);
BEBELM_API int bebelm_gguf_get_u32_array(const bebelm_gguf* g, const char* key, uint32_t* out, size_t cap,
                                         size_t* len);
/* An array's element type and length, and its i-th string (get_str_array, src/gguf.rs:248-262). */
BEBELM_API int bebelm_gguf_array_len(const bebelm_gguf* g, const char* key, int* elem_type, size_t* len);
BEBELM_API int bebelm_gguf_get_str_at(const bebelm_gguf* g, const char* key, size_t i, const char** s,
                                      size_t* len);
/* config::validate (src/config.rs:50-96): BEBELM_ERR_FORMAT unless the metadata is
 * LFM2.5-8B-A1B's (architecture, sizes, rope base, eps, the kv-head schedule). */
BEBELM_API int bebelm_gguf_validate(const bebelm_gguf* g);
/* The attention weights of block `block` (0..23; attention blocks 2, 6, 10, 14, 18, 21)
 * by their GGUF names blk.N.attn_{q,k,v,output}.weight and blk.N.attn_{q,k}_norm.weight
 * (src/model.rs:228-233, 434-439, 454), uploaded by bebelm_attn_weights_create. */
BEBELM_API int bebelm_attn_weights_from_gguf(const bebelm_gguf* g, int block, int device,
                                             bebelm_attn_weights** out);
/* The logits head from token_embd.weight and token_embd_norm.weight (src/model.rs:379-388),
 * uploaded by bebelm_head_create. */
BEBELM_API int bebelm_head_from_gguf(const bebelm_gguf* g, int device, bebelm_head** out);

#ifdef __cplusplus
}
#endif
#endif /* BEBELM_ATTN_H */
