// Host runtime behind the C-ABI of include/bebelm_attn.h: page pool and
// sequence-window bookkeeping (the device replacement of src/cache.rs), host /
// device staging, and the launch sequences of the fused calls.
#include <algorithm>
#include <atomic>
#include <climits>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <condition_variable>
#include <mutex>
#include <string>
#include <thread>
#include <unordered_map>
#include <initializer_list>
#include <vector>

#include <unistd.h>

#include "../../include/bebelm_attn.h"
#include "internal.h"

using namespace bebelm;

// ------------------------------------------------------------------ errors --
static thread_local std::string g_err;

static int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_err = buf;
    return code;
}

int bebelm::set_last_error(int code, const char* msg) {
    g_err = msg;
    return code;
}

#define CUDA_TRY(x)                                                                          \
    do {                                                                                     \
        cudaError_t e_ = (x);                                                                \
        if (e_ != cudaSuccess)                                                               \
            return fail(e_ == cudaErrorMemoryAllocation ? BEBELM_ERR_OOM : BEBELM_ERR_CUDA,  \
                        "%s failed: %s (%s:%d)", #x, cudaGetErrorString(e_), __FILE__, __LINE__); \
    } while (0)

#define TRY(x)                 \
    do {                       \
        int rc_ = (x);         \
        if (rc_ != 0) return rc_; \
    } while (0)

namespace {

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

int check_device(int dev) {
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess || n == 0)
        return fail(BEBELM_ERR_NO_DEVICE, "no CUDA device visible (%s)", cudaGetErrorString(e));
    if (dev < 0 || dev >= n) return fail(BEBELM_ERR_INVALID, "device %d out of range [0,%d)", dev, n);
    int major = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    if (major != 10)
        return fail(BEBELM_ERR_NO_DEVICE, "device %d is sm_%d0, this library is built for sm_100a", dev, major);
    return 0;
}

int current_device(int* dev) {
    CUDA_TRY(cudaGetDevice(dev));
    return check_device(*dev);
}

// Growable device buffer.
struct DevBuf {
    void* p = nullptr;
    size_t bytes = 0;
    int ensure(size_t need, bool zero = false, cudaStream_t s = 0) {
        if (need <= bytes) return 0;
        // a buffer that has to grow gets half as much again on top: scratch that follows a
        // growing window (split partials of a decode step whose sequences lengthen) then grows
        // a few times per run, not every few steps — each regrowth waits for the stream
        size_t n = std::max<size_t>(need, 256);
        if (p) {
            n = std::max(n, bytes + bytes / 2);
            cudaStreamSynchronize(s);
            cudaFree(p);
            p = nullptr;
            bytes = 0;
        }
        CUDA_TRY(cudaMalloc(&p, n));
        bytes = n;
        if (zero) CUDA_TRY(cudaMemsetAsync(p, 0, n, s));
        return 0;
    }
    void release() {
        if (p) cudaFree(p);
        p = nullptr;
        bytes = 0;
    }
    template <class T> T* as() const { return static_cast<T*>(p); }
};

// Growable pinned host buffer, also mapped into the device's address space (d): a kernel
// may store a small result straight into it instead of the host copying it back.
struct PinBuf {
    void* p = nullptr;
    void* d = nullptr;
    size_t bytes = 0;
    int ensure(size_t need) {
        if (need <= bytes) return 0;
        if (p) cudaFreeHost(p);
        p = d = nullptr;
        bytes = 0;
        size_t n = std::max<size_t>(need, 4096);
        CUDA_TRY(cudaHostAlloc(&p, n, cudaHostAllocMapped | cudaHostAllocPortable));
        bytes = n;
        CUDA_TRY(cudaHostGetDevicePointer(&d, p, 0));
        return 0;
    }
    void release() {
        if (p) cudaFreeHost(p);
        p = d = nullptr;
        bytes = 0;
    }
    template <class T> T* as() const { return static_cast<T*>(p); }
};

// A pool's error word: pinned host memory mapped into the device. A kernel whose bounded
// wait gives up stores its code there (a plain store); the host reads it after
// synchronising, without a copy.
struct ErrWord {
    int* h = nullptr;  // host address
    int* d = nullptr;  // device address of the same word
    int ensure() {
        if (h) return 0;
        void* p = nullptr;
        CUDA_TRY(cudaHostAlloc(&p, 64, cudaHostAllocMapped | cudaHostAllocPortable));
        h = static_cast<int*>(p);
        *h = 0;
        void* dp = nullptr;
        CUDA_TRY(cudaHostGetDevicePointer(&dp, p, 0));
        d = static_cast<int*>(dp);
        return 0;
    }
    int read() const { return *reinterpret_cast<volatile int*>(h); }
    void clear() { *reinterpret_cast<volatile int*>(h) = 0; }
    void release() {
        if (h) cudaFreeHost(h);
        h = d = nullptr;
    }
};

}  // namespace

// Large copies between caller memory and the pinned staging buffer run on a few host threads:
// one thread's memcpy is slower than the host link, and a prefill of thousands of tokens moves
// tens of MB each way. The calling thread takes a share; `copy` returns once all are done.
struct HostCopier {
    static constexpr size_t kMinParallel = 1 << 20;
    std::vector<std::thread> th;
    std::mutex mu, run;
    std::condition_variable cv, cv_done;
    char* dst = nullptr;
    const char* src = nullptr;
    size_t n = 0;
    int parts = 0;
    std::atomic<int> next{0}, done{0};
    unsigned long long gen = 0;

    pid_t owner = 0;  // the process whose threads these are (a forked child has none of them)

    // Created on first use and never destroyed: the idle workers end with the process, and no
    // exit-time join can wait on threads that a forked child does not have.
    static HostCopier& get() {
        static HostCopier* c = new HostCopier();
        return *c;
    }
    HostCopier() : owner(getpid()) {
        const unsigned hc = std::thread::hardware_concurrency();
        const int k = (int)std::min(7u, hc > 2 ? hc / 2 : 0u);
        for (int i = 0; i < k; ++i) th.emplace_back([this] { loop(); });
    }
    void work() {
        for (;;) {
            const int i = next.fetch_add(1);
            if (i >= parts) return;
            const size_t a = n * (size_t)i / (size_t)parts, b = n * (size_t)(i + 1) / (size_t)parts;
            std::memcpy(dst + a, src + a, b - a);
            if (done.fetch_add(1) + 1 == parts) {
                std::lock_guard<std::mutex> lk(mu);
                cv_done.notify_all();
            }
        }
    }
    void loop() {
        unsigned long long seen = 0;
        for (;;) {
            {
                std::unique_lock<std::mutex> lk(mu);
                cv.wait(lk, [&] { return gen != seen; });
                seen = gen;
            }
            work();
        }
    }
    void copy(void* d, const void* sp, size_t bytes) {
        if (bytes < kMinParallel || th.empty() || getpid() != owner) {
            std::memcpy(d, sp, bytes);
            return;
        }
        std::lock_guard<std::mutex> one(run);  // one parallel copy at a time
        {
            std::lock_guard<std::mutex> lk(mu);
            dst = static_cast<char*>(d);
            src = static_cast<const char*>(sp);
            n = bytes;
            parts = 2 * ((int)th.size() + 1);
            done = 0;
            next = 0;
            ++gen;
        }
        cv.notify_all();
        work();
        std::unique_lock<std::mutex> lk(mu);
        cv_done.wait(lk, [&] { return done.load() >= parts; });
    }
};

// Host-link transfers of a large staged call go in chunks of this size: the copy of chunk i
// between caller memory and the pinned buffer overlaps the DMA of its neighbour.
constexpr size_t kStageChunk = 4u << 20;
constexpr int kStageEvents = 8;

// Small host-to-device uploads (page-table entries, sequence descriptors) go through a
// ring of pinned slots: a copy from pinned memory is truly asynchronous, whereas one from
// pageable memory is staged by the runtime and can hold the host to the GPU's pace. A slot
// is reused only after the event recorded behind its last copy has completed.
struct UploadRing {
    static constexpr int kSlots = 16;
    static constexpr size_t kSlotBytes = 64 * 1024;
    char* pin = nullptr;
    cudaEvent_t done[kSlots] = {};
    int next = 0;

    // Enqueues a copy of `bytes` from src to the device address dst on stream s.
    cudaError_t copy(void* dst, const void* src, size_t bytes, cudaStream_t s) {
        if (bytes > kSlotBytes) return cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, s);
        if (!pin) {
            cudaError_t e = cudaHostAlloc(reinterpret_cast<void**>(&pin), kSlots * kSlotBytes, cudaHostAllocDefault);
            if (e != cudaSuccess) return e;
            for (int i = 0; i < kSlots; ++i) {
                e = cudaEventCreateWithFlags(&done[i], cudaEventDisableTiming);
                if (e != cudaSuccess) return e;
            }
        }
        const int i = next;
        next = (next + 1) % kSlots;
        cudaError_t e = cudaEventSynchronize(done[i]);  // the slot's previous copy has been read
        if (e != cudaSuccess) return e;
        std::memcpy(pin + (size_t)i * kSlotBytes, src, bytes);
        e = cudaMemcpyAsync(dst, pin + (size_t)i * kSlotBytes, bytes, cudaMemcpyHostToDevice, s);
        if (e != cudaSuccess) return e;
        return cudaEventRecord(done[i], s);
    }
    void release() {
        for (int i = 0; i < kSlots; ++i)
            if (done[i]) cudaEventDestroy(done[i]);
        if (pin) cudaFreeHost(pin);
        pin = nullptr;
    }
};

// -------------------------------------------------------------------- pool --
struct bebelm_kv_pool {
    int device = 0, n_layers = 0, n_kv = 0, head_dim = 64, page_tokens = 64, dtype = BEBELM_F32;
    size_t n_pages = 0, page_bytes = 0, block_bytes = 0;
    char* mem = nullptr;
    std::vector<int> free_list;  // physical pages not in any window
    int num_sms = 148;
    int n_seqs = 0;              // live sequences drawing from this pool
    // scratch shared by every call on this pool's sequences (stream-ordered)
    DevBuf io, qn, part, counters, seqdesc, pf, q8, proj, sample;
    ErrWord err;
    PinBuf pin;
    cudaEvent_t out_ev[kStageEvents] = {};  // chunks of a large output copied back
    UploadRing uploads;
    // a second stream for work that may run beside the caller's (forked and joined with events
    // inside one call, so the call stays ordered on the caller's stream)
    cudaStream_t side = nullptr;
    cudaEvent_t ev_fork = nullptr, ev_join = nullptr;
    const void* last_plan = nullptr;  // the step plan of the last decode launch, if it was one
    unsigned long long last_capture = 0;  // the stream capture that launch was recorded in (0: none)
    std::vector<DecodeSeq> h_desc;
    // cache slots written by the most recent library kernel on this pool: a decode
    // launched next copies pages below these before its griddepcontrol.wait
    struct Written {
        const bebelm_kv* kv;
        int layer;
        long long slot_lo;
    };
    std::vector<Written> last_writes;

    PoolView view(int layer) const {
        PoolView v;
        v.base = mem;
        v.page_bytes = page_bytes;
        v.layer_off = (size_t)layer * 2 * block_bytes;
        v.block_bytes = block_bytes;
        v.kind = dtype == BEBELM_BF16 ? kElemBF16 : dtype == BEBELM_FP8_E4M3 ? kElemFP8 : kElemF32;
        return v;
    }
};

struct bebelm_kv {
    bebelm_kv_pool* pool = nullptr;
    bool owns_pool = false;
    size_t max_context = 0;
    int cap = 0;                  // ring entries (logical pages held at most)
    int* d_table = nullptr;       // device copy of the ring
    std::vector<int> table;       // ring: logical page L -> physical table[L % cap]
    long long lo = 0, hi = 0;     // allocated logical pages [lo, hi)
    std::vector<long long> base, len;  // per layer window: slots [base, base+len)
    size_t pos = 0;
    int plans = 0;                // open step plans: the device owns the window state meanwhile
};

namespace {

int upload_table(bebelm_kv* kv, long long L0, long long L1, cudaStream_t s) {
    // ring entries of logical pages [L0, L1), copied through the pool's pinned upload ring
    // (the bytes are captured when the copy is enqueued, so later host edits cannot race)
    for (long long L = L0; L < L1;) {
        int i0 = (int)(L % kv->cap);
        long long n = std::min<long long>(L1 - L, kv->cap - i0);
        CUDA_TRY(kv->pool->uploads.copy(kv->d_table + i0, kv->table.data() + i0, sizeof(int) * n, s));
        L += n;
    }
    return 0;
}

// Make room for t more positions of `layer`; returns the logical slot of the first.
int reserve(bebelm_kv* kv, int layer, size_t t, long long* slot0, cudaStream_t s) {
    long long b = kv->base[layer], n = kv->len[layer];
    if (n == 0 && b < kv->lo * kPageTokens) b = kv->lo * kPageTokens;
    const long long s0 = b + n, s_end = s0 + (long long)t;
    const long long need_hi = (s_end + kPageTokens - 1) / kPageTokens;
    if (need_hi - kv->lo > kv->cap)
        return fail(BEBELM_ERR_CAPACITY,
                    "layer %d window would hold %lld positions; this cache holds at most %zu (+%d): "
                    "evict_front first",
                    layer, n + (long long)t, kv->max_context, kPageTokens);
    const long long add = std::max<long long>(0, need_hi - kv->hi);
    if ((size_t)add > kv->pool->free_list.size())
        return fail(BEBELM_ERR_OOM, "page pool exhausted: need %lld pages, %zu free", add,
                    kv->pool->free_list.size());
    const long long old_hi = kv->hi;
    for (long long L = kv->hi; L < need_hi; ++L) {
        kv->table[L % kv->cap] = kv->pool->free_list.back();
        kv->pool->free_list.pop_back();
    }
    if (need_hi > kv->hi) kv->hi = need_hi;
    if (add) TRY(upload_table(kv, old_hi, kv->hi, s));
    kv->base[layer] = b;
    kv->len[layer] = n + (long long)t;
    *slot0 = s0;
    return 0;
}

void release_pages_below(bebelm_kv* kv, long long new_lo) {
    for (long long L = kv->lo; L < new_lo; ++L) kv->pool->free_list.push_back(kv->table[L % kv->cap]);
    kv->lo = new_lo;
}

void recompute_lo(bebelm_kv* kv) {
    long long new_lo = kv->hi;
    for (size_t l = 0; l < kv->len.size(); ++l)
        if (kv->len[l] > 0) new_lo = std::min(new_lo, kv->base[l] / kPageTokens);
    if (new_lo > kv->lo) release_pages_below(kv, new_lo);
}

int validate_kv(const bebelm_kv* kv) {
    if (!kv || !kv->pool) return fail(BEBELM_ERR_INVALID, "null cache handle");
    if (kv->plans > 0)
        return fail(BEBELM_ERR_INVALID, "the cache has %d open step plan(s): finish them first", kv->plans);
    return 0;
}

int validate_layer(const bebelm_kv* kv, int layer) {
    TRY(validate_kv(kv));
    if (layer < 0 || layer >= kv->pool->n_layers)
        return fail(BEBELM_ERR_INVALID, "layer %d out of range [0,%d)", layer, kv->pool->n_layers);
    return 0;
}

int pool_create(int n_layers, int n_kv_heads, int head_dim, size_t n_pages, int page_tokens, int dtype,
                int device, bebelm_kv_pool** out) {
    if (!out) return fail(BEBELM_ERR_INVALID, "out is null");
    *out = nullptr;
    if (n_layers <= 0 || n_kv_heads <= 0 || n_pages == 0)
        return fail(BEBELM_ERR_INVALID, "n_layers, n_kv_heads and n_pages must be positive");
    if (head_dim != kHeadDim) return fail(BEBELM_ERR_UNSUPPORTED, "cache head_dim must be 64 (got %d)", head_dim);
    if (page_tokens != kPageTokens)
        return fail(BEBELM_ERR_UNSUPPORTED, "page_tokens must be 64 (got %d)", page_tokens);
    if (dtype != BEBELM_F32 && dtype != BEBELM_BF16 && dtype != BEBELM_FP8_E4M3)
        return fail(BEBELM_ERR_UNSUPPORTED, "cache dtype must be BEBELM_F32, BEBELM_BF16 or BEBELM_FP8_E4M3");
    if (n_pages > (size_t)INT32_MAX) return fail(BEBELM_ERR_INVALID, "too many pages");
    TRY(check_device(device));
    DeviceGuard g(device);
    auto* P = new bebelm_kv_pool();
    P->device = device;
    P->n_layers = n_layers;
    P->n_kv = n_kv_heads;
    P->n_pages = n_pages;
    P->dtype = dtype;
    P->block_bytes = (size_t)n_kv_heads * kPageRowFloats * (dtype == BEBELM_F32 ? 4 : dtype == BEBELM_BF16 ? 2 : 1);
    P->page_bytes = (size_t)n_layers * 2 * P->block_bytes;
    cudaDeviceGetAttribute(&P->num_sms, cudaDevAttrMultiProcessorCount, device);
    const size_t bytes = n_pages * P->page_bytes;
    cudaError_t e = cudaMalloc(&P->mem, bytes);
    if (e != cudaSuccess) {
        delete P;
        return fail(BEBELM_ERR_OOM, "cudaMalloc of %zu bytes for the page pool failed: %s", bytes,
                    cudaGetErrorString(e));
    }
    // zero once so masked rows of a partly filled page are finite
    e = cudaMemset(P->mem, 0, bytes);
    if (e == cudaSuccess) {
        int rc = P->err.ensure();
        if (rc) {
            cudaFree(P->mem);
            delete P;
            return rc;
        }
        e = cudaDeviceSynchronize();
    }
    if (e != cudaSuccess) {
        cudaFree(P->mem);
        delete P;
        return fail(BEBELM_ERR_CUDA, "pool initialisation failed: %s", cudaGetErrorString(e));
    }
    P->free_list.reserve(n_pages);
    for (size_t i = n_pages; i-- > 0;) P->free_list.push_back((int)i);
    *out = P;
    return 0;
}

void pool_free(bebelm_kv_pool* P) {
    DeviceGuard g(P->device);
    cudaDeviceSynchronize();
    P->uploads.release();
    if (P->side) cudaStreamDestroy(P->side);
    if (P->ev_fork) cudaEventDestroy(P->ev_fork);
    if (P->ev_join) cudaEventDestroy(P->ev_join);
    P->side = nullptr;
    P->ev_fork = P->ev_join = nullptr;
    cudaFree(P->mem);
    P->io.release();
    P->qn.release();
    P->part.release();
    P->counters.release();
    P->seqdesc.release();
    P->pf.release();
    P->q8.release();
    P->proj.release();
    P->sample.release();
    P->err.release();
    P->pin.release();
    for (cudaEvent_t& e : P->out_ev)
        if (e) cudaEventDestroy(e);
    delete P;
}

int seq_create(bebelm_kv_pool* P, size_t max_context, bool owns, bebelm_kv** out) {
    if (!out) return fail(BEBELM_ERR_INVALID, "out is null");
    *out = nullptr;
    if (max_context == 0) return fail(BEBELM_ERR_INVALID, "max_context must be positive");
    DeviceGuard g(P->device);
    auto* kv = new bebelm_kv();
    kv->pool = P;
    kv->owns_pool = owns;
    kv->max_context = max_context;
    kv->cap = (int)((max_context + kPageTokens - 1) / kPageTokens + 2);
    kv->table.assign(kv->cap, 0);
    kv->base.assign(P->n_layers, 0);
    kv->len.assign(P->n_layers, 0);
    cudaError_t e = cudaMalloc(&kv->d_table, sizeof(int) * kv->cap);
    if (e == cudaSuccess) e = cudaMemset(kv->d_table, 0, sizeof(int) * kv->cap);
    if (e != cudaSuccess) {
        delete kv;
        return fail(BEBELM_ERR_OOM, "page table allocation failed: %s", cudaGetErrorString(e));
    }
    P->n_seqs++;
    *out = kv;
    return 0;
}

}  // namespace

namespace {

struct Window {
    const bebelm_kv* kv;
    long long base;
    long long len;
    long long new_slot;  // appended by this launch (fused step) or -1
    long long pos;       // RoPE position of the query (fused step)
};

// Inputs of a fused decode step: raw q (and the appended token's raw k, v), gains.
struct FusedStep {
    const float* q_raw;
    const float* k_new;
    const float* v_new;
    const float* q_gain;
    const float* k_gain;
    float theta_scale;
    float eps;
};

// The output range of the last decode launch on each stream. Only decode grids launch as
// programmatic dependents, so a decode grid can overlap nothing but the previous decode grid on
// its stream, and that grid passed its own griddepcontrol.wait (everything before it complete)
// before it let this one start: inputs outside its output were complete when this grid began.
struct OutRange {
    const char* p = nullptr;
    size_t n = 0;  // SIZE_MAX: unknown (e.g. stores to peers), overlaps everything
};
std::mutex g_last_out_mu;
std::unordered_map<cudaStream_t, OutRange> g_last_out;

void record_decode_out(cudaStream_t s, const void* out, size_t bytes) {
    std::lock_guard<std::mutex> lk(g_last_out_mu);
    g_last_out[s] = OutRange{static_cast<const char*>(out), bytes};
}

// the running host call's inputs are copied to the device by a kernel (see stage_in)
thread_local bool g_inputs_staged = false;

bool inputs_clear_of_last_out(cudaStream_t s, std::initializer_list<std::pair<const void*, size_t>> ins) {
    std::lock_guard<std::mutex> lk(g_last_out_mu);
    auto it = g_last_out.find(s);
    if (it == g_last_out.end()) return true;  // no decode grid before this one on the stream
    const OutRange r = it->second;
    if (r.n == SIZE_MAX) return false;
    for (const auto& in : ins) {
        const char* p = static_cast<const char*>(in.first);
        if (p && p < r.p + r.n && r.p < p + in.second) return false;
    }
    return true;
}

// Split size cap of batched decode (pages per CTA). Config 4 (64 sequences, 1k-16k positions):
// 8, 32 and 64 pages gave 0.545, 0.436 and 0.434 ms per step; small caps make thousands of
// short CTAs, each paying its prologue and its share of the merge.
#ifndef BEBELM_BATCH_PAGES_PER_SPLIT
#define BEBELM_BATCH_PAGES_PER_SPLIT 32
#endif
constexpr long long kBatchMaxPagesPerSplit = BEBELM_BATCH_PAGES_PER_SPLIT;

void pick_heads_per_cta(int group, int* hpc, int* n_sub) {
    int h = group % 4 == 0 ? 4 : group % 3 == 0 ? 3 : group % 2 == 0 ? 2 : 1;
    *hpc = h;
    *n_sub = group / h;
}

long long dep_slot_for(const bebelm_kv_pool* P, const bebelm_kv* kv, int layer) {
    long long d = LLONG_MAX;
    for (const auto& w : P->last_writes)
        if (w.kv == kv && w.layer == layer) d = std::min(d, w.slot_lo);
    return d;
}

// Split-K decode of one query per window. out: [n_windows][n_heads][64] device. The
// query is d_q (normed+roped, [n][n_heads][64]) or, for a fused step, fused->q_raw.
// Where a fused all-gather sends the final outputs (one window only): every rank's landing zone.
struct PeerTarget {
    unsigned long long* const* bufs;  // every rank's landing zone (tagged words)
    int world, rank;
    const unsigned long long* epoch;  // the group's device epoch word
};

int run_decode(bebelm_kv_pool* P, const std::vector<Window>& wins, int layer, int n_heads, const float* d_q,
               float* d_out, float scale, const FusedStep* fused, cudaStream_t s, const PeerTarget* peer = nullptr) {
    const int n = (int)wins.size();
    if (n == 0) return 0;
    const int group = n_heads / P->n_kv;
    int hpc, n_sub;
    pick_heads_per_cta(group, &hpc, &n_sub);
    const int NY = P->n_kv * n_sub;
    long long total_units = 0;
    std::vector<long long> npages(n);
    for (int i = 0; i < n; ++i) {
        const Window& w = wins[i];
        npages[i] = w.len > 0 ? (w.base + w.len - 1) / kPageTokens - w.base / kPageTokens + 1 : 0;
        total_units += npages[i] * NY;
    }
    const long long target = (long long)P->num_sms * 2;  // two resident CTAs per SM
    long long per = std::max<long long>(1, (total_units + target - 1) / target);
    if (n > 1) per = std::min<long long>(per, kBatchMaxPagesPerSplit);  // uneven sequences: more, smaller splits
    per = std::min<long long>(per, kDecodeMaxPagesPerSplit);
    P->h_desc.resize(n);
    int total_splits = 0;
    for (int i = 0; i < n; ++i) {
        DecodeSeq& d = P->h_desc[i];
        d.table = wins[i].kv->d_table;
        d.cap = wins[i].kv->cap;
        d.len = (int)wins[i].len;
        d.base = wins[i].base;
        d.split0 = total_splits;
        d.n_splits = (int)std::max<long long>(1, (npages[i] + per - 1) / per);
        d.new_slot = fused ? wins[i].new_slot : -1;
        d.pos = wins[i].pos;
        d.dep_slot = dep_slot_for(P, wins[i].kv, layer);
        total_splits += d.n_splits;
    }
    // room for one more split per sequence: a growing window then crosses into a new split (and
    // a regrowth, which waits for the stream) only once per `per` pages of steps
    const size_t part_splits = (size_t)total_splits + (n > 1 ? (size_t)n : 0);
    TRY(P->part.ensure(sizeof(float) * part_splits * NY * hpc * (kHeadDim + 2), false, s));
    TRY(P->counters.ensure(sizeof(unsigned) * (size_t)n * NY, true, s));
    DecodeArgs a{};
    if (n == 1) {
        a.one = P->h_desc[0];
    } else {
        TRY(P->seqdesc.ensure(sizeof(DecodeSeq) * n, false, s));
        CUDA_TRY(P->uploads.copy(P->seqdesc.p, P->h_desc.data(), sizeof(DecodeSeq) * n, s));
        a.seqs = P->seqdesc.as<DecodeSeq>();
    }
    a.n_seqs = n;
    a.pv = P->view(layer);
    a.q = d_q;
    if (fused) {
        a.q_raw = fused->q_raw;
        a.k_new = fused->k_new;
        a.v_new = fused->v_new;
        a.q_gain = fused->q_gain;
        a.k_gain = fused->k_gain;
        a.theta_scale = fused->theta_scale;
        a.eps = fused->eps;
        const size_t nq = (size_t)n * n_heads * kHeadDim * 4, nkv = (size_t)n * P->n_kv * kHeadDim * 4;
        // inputs staged from host memory by a copy kernel are complete only after the wait
        a.early_inputs = !g_inputs_staged && !peer && inputs_clear_of_last_out(s, {{fused->q_raw, nq}, {fused->k_new, nkv},
                                                               {fused->v_new, nkv}, {fused->q_gain, 4 * kHeadDim},
                                                               {fused->k_gain, 4 * kHeadDim}});
    }
    a.out = d_out;
    a.part_acc = P->part.as<float>();
    a.part_ml = a.part_acc + (size_t)total_splits * NY * hpc * kHeadDim;
    a.counters = P->counters.as<unsigned>();
    a.err = P->err.d;
    a.n_heads = n_heads;
    a.n_kv = P->n_kv;
    a.group = group;
    a.hpc = hpc;
    a.n_sub = n_sub;
    a.pages_per_split = (int)per;
    a.total_splits = total_splits;
    a.scale_log2 = scale * 1.4426950408889634f;
    a.pdl = 1;
    if (g_expire_waits > 0) {  // test hook (bebelm_debug_expire_next_wait)
        a.expire_wait = 1;
        --g_expire_waits;
    }
    if (peer) {
        a.peer_bufs = peer->bufs;
        a.peer_world = peer->world;
        a.peer_rank = peer->rank;
        a.peer_epoch = peer->epoch;
    }
    CUDA_TRY(launch_decode(a, s));
    record_decode_out(s, d_out, peer ? SIZE_MAX : (size_t)n * n_heads * kHeadDim * 4);
    P->last_plan = nullptr;
    P->last_writes.clear();
    if (fused)
        for (int i = 0; i < n; ++i)
            if (wins[i].new_slot >= 0) P->last_writes.push_back({wins[i].kv, layer, wins[i].new_slot});
    return 0;
}

// Copies host inputs into pinned staging and then into the pool's device io buffer.
struct Stage {
    const void* src;
    size_t bytes;
    void** dev;  // receives the device address
};

thread_local size_t g_pin_out_off = 0;   // set by stage_in, read by stage_out (calls are host-synchronous)
// Host inputs up to this size reach the device through a copy kernel rather than a DMA copy:
// the decode grid launched behind it overlaps its prologue with the copy (programmatic
// dependent launch), where a cudaMemcpyAsync before it would finish first.
constexpr size_t kKernelStageBytes = 64 * 1024;
thread_local bool g_pin_out_direct = false;  // the output was stored straight into the pinned buffer

// Outputs up to this size are stored by the kernel straight into the mapped pinned buffer
// (over the host link, as the copy back would go); larger ones are copied back once.
constexpr size_t kDirectOutBytes = 64 * 1024;

int stage_in(bebelm_kv_pool* P, Stage* st, int n, size_t out_bytes, void** d_out, cudaStream_t s) {
    size_t total = 0;
    for (int i = 0; i < n; ++i) total += (st[i].bytes + 255) & ~size_t(255);
    const size_t out_off = total;
    total += ((out_bytes + 255) & ~size_t(255)) + 256;
    TRY(P->io.ensure(total, false, s));
    TRY(P->pin.ensure(total));
    g_inputs_staged = out_off > 0 && out_off <= kKernelStageBytes;
    size_t off = 0;
    for (int i = 0; i < n; ++i) {
        *st[i].dev = st[i].src ? P->io.as<char>() + off : nullptr;
        if (st[i].src && st[i].bytes) {
            char* pin = P->pin.as<char>() + off;
            if (g_inputs_staged) {
                std::memcpy(pin, st[i].src, st[i].bytes);
            } else {  // large: chunk by chunk, each DMA overlapping the next chunk's host copy
                for (size_t c = 0; c < st[i].bytes; c += kStageChunk) {
                    const size_t len = std::min(kStageChunk, st[i].bytes - c);
                    HostCopier::get().copy(pin + c, static_cast<const char*>(st[i].src) + c, len);
                    CUDA_TRY(cudaMemcpyAsync(P->io.as<char>() + off + c, pin + c, len, cudaMemcpyHostToDevice, s));
                }
            }
        }
        off += (st[i].bytes + 255) & ~size_t(255);
    }
    if (g_inputs_staged) CUDA_TRY(launch_stage_copy(P->io.p, P->pin.d, out_off, s));
    g_pin_out_direct = out_bytes <= kDirectOutBytes;
    if (d_out) *d_out = (g_pin_out_direct ? static_cast<char*>(P->pin.d) : P->io.as<char>()) + out_off;
    g_pin_out_off = out_off;
    return 0;
}

// Zeroes the split counters of the no-allocation decode on `dev` (if that path was ever set up
// there): a decode CTA that gave up on a wait left its counter short.
void clear_noalloc_counters(int dev, cudaStream_t s);

// Waits for the call's work, surfaces a device-side timeout recorded by a kernel, and
// delivers the output to the caller's host memory (from the pinned buffer, after copying
// it there unless the kernel stored it there directly).
int stage_out(bebelm_kv_pool* P, const void* d_src, void* h_dst, size_t bytes, cudaStream_t s) {
    g_inputs_staged = false;
    char* pin = P->pin.as<char>() + g_pin_out_off;
    if (bytes > kStageChunk && !g_pin_out_direct) {
        // large: chunks copied back behind events, each delivered while the next one crosses
        const size_t chunk = std::max(kStageChunk, (bytes + kStageEvents - 1) / kStageEvents);
        const int nc = (int)((bytes + chunk - 1) / chunk);
        for (int i = 0; i < nc; ++i) {
            if (!P->out_ev[i]) CUDA_TRY(cudaEventCreateWithFlags(&P->out_ev[i], cudaEventDisableTiming));
            const size_t c = (size_t)i * chunk, len = std::min(chunk, bytes - c);
            CUDA_TRY(cudaMemcpyAsync(pin + c, static_cast<const char*>(d_src) + c, len, cudaMemcpyDeviceToHost, s));
            CUDA_TRY(cudaEventRecord(P->out_ev[i], s));
        }
        CUDA_TRY(cudaEventSynchronize(P->out_ev[0]));  // every kernel of the call has completed
        if (P->err.read() == 0) {
            for (int i = 0; i < nc; ++i) {
                const size_t c = (size_t)i * chunk, len = std::min(chunk, bytes - c);
                if (i) CUDA_TRY(cudaEventSynchronize(P->out_ev[i]));
                HostCopier::get().copy(static_cast<char*>(h_dst) + c, pin + c, len);
            }
            bytes = 0;  // delivered
        }
    } else if (bytes && !g_pin_out_direct) {
        CUDA_TRY(cudaMemcpyAsync(pin, d_src, bytes, cudaMemcpyDeviceToHost, s));
    }
    CUDA_TRY(cudaStreamSynchronize(s));
    const int derr = P->err.read();
    if (derr) {
        P->err.clear();
        if (P->counters.p) cudaMemsetAsync(P->counters.p, 0, P->counters.bytes, s);
        clear_noalloc_counters(P->device, s);
        cudaStreamSynchronize(s);
        return fail(BEBELM_ERR_TIMEOUT, "a device-side wait timed out (code %d); outputs are invalid", derr);
    }
    if (bytes) std::memcpy(h_dst, pin, bytes);
    return 0;
}

float theta_scale_of(float theta, int head_dim) {
    // src/kernels/rope.rs:19: freq_base.powf(-2.0 / d as f32), evaluated with the host libm
    return powf(theta, -2.0f / (float)head_dim);
}

}  // namespace

namespace {

// Staging for calls that have no pool (the drop-ins): one per device, guarded by a mutex.
std::mutex g_scratch_mu;
bebelm_kv_pool* g_scratch[64] = {};

int scratch_pool(int dev, bebelm_kv_pool** out) {
    if (dev < 0 || dev >= 64) return fail(BEBELM_ERR_INVALID, "device %d unsupported", dev);
    if (!g_scratch[dev]) {
        auto* P = new bebelm_kv_pool();
        P->device = dev;
        int rc = P->err.ensure();
        if (rc) {
            delete P;
            return rc;
        }
        cudaDeviceGetAttribute(&P->num_sms, cudaDevAttrMultiProcessorCount, dev);
        g_scratch[dev] = P;
    }
    *out = g_scratch[dev];
    return 0;
}

cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

int check_mem(int mem) {
    if (mem != BEBELM_MEM_HOST && mem != BEBELM_MEM_DEVICE)
        return fail(BEBELM_ERR_INVALID, "mem must be BEBELM_MEM_HOST or BEBELM_MEM_DEVICE (got %d)", mem);
    return 0;
}

int check_geometry(int n_heads, int n_kv) {
    if (n_heads <= 0 || n_kv <= 0 || n_heads % n_kv)
        return fail(BEBELM_ERR_INVALID, "n_heads (%d) must be a positive multiple of n_kv_heads (%d)", n_heads, n_kv);
    return 0;
}

}  // namespace

extern "C" {

int bebelm_abi_version(void) { return BEBELM_ABI_VERSION; }

int bebelm_last_error(char* buf, size_t n) {
    if (!buf || !n) return BEBELM_ERR_INVALID;
    std::snprintf(buf, n, "%s", g_err.c_str());
    return 0;
}

int bebelm_device_count(int* n) {
    if (!n) return fail(BEBELM_ERR_INVALID, "n is null");
    *n = 0;
    int total = 0;
    if (cudaGetDeviceCount(&total) != cudaSuccess) return 0;
    for (int d = 0; d < total; ++d) {
        int major = 0;
        cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, d);
        if (major == 10) ++*n;
    }
    return 0;
}

// ------------------------------------------------------------------ pool --
int bebelm_kv_pool_create(int n_layers, int n_kv_heads, int head_dim, size_t n_pages, int page_tokens, int dtype,
                          int device, bebelm_kv_pool** out) {
    return pool_create(n_layers, n_kv_heads, head_dim, n_pages, page_tokens, dtype, device, out);
}

int bebelm_kv_pool_destroy(bebelm_kv_pool* pool) {
    if (!pool) return fail(BEBELM_ERR_INVALID, "null pool");
    if (pool->n_seqs) return fail(BEBELM_ERR_INVALID, "pool still has %d live sequences", pool->n_seqs);
    pool_free(pool);
    return 0;
}

int bebelm_kv_pool_free_pages(const bebelm_kv_pool* pool, size_t* out) {
    if (!pool || !out) return fail(BEBELM_ERR_INVALID, "null argument");
    *out = pool->free_list.size();
    return 0;
}

// ----------------------------------------------------------------- cache --
int bebelm_kv_create(int n_layers, int n_kv_heads, int head_dim, size_t max_context, int page_tokens, int dtype,
                     int device, bebelm_kv** out) {
    if (!out) return fail(BEBELM_ERR_INVALID, "out is null");
    *out = nullptr;
    if (max_context == 0) return fail(BEBELM_ERR_INVALID, "max_context must be positive");
    const size_t pages = (max_context + kPageTokens - 1) / kPageTokens + 2;
    bebelm_kv_pool* P = nullptr;
    TRY(pool_create(n_layers, n_kv_heads, head_dim, pages, page_tokens, dtype, device, &P));
    int rc = seq_create(P, max_context, true, out);
    if (rc) pool_free(P);
    return rc;
}

int bebelm_kv_create_in_pool(bebelm_kv_pool* pool, size_t max_context, bebelm_kv** out) {
    if (!pool) return fail(BEBELM_ERR_INVALID, "null pool");
    return seq_create(pool, max_context, false, out);
}

int bebelm_kv_destroy(bebelm_kv* kv) {
    if (!kv) return 0;
    if (kv->plans > 0)
        return fail(BEBELM_ERR_INVALID, "the cache has %d open step plan(s): finish them first", kv->plans);
    bebelm_kv_pool* P = kv->pool;
    {
        DeviceGuard g(P->device);
        cudaDeviceSynchronize();  // kernels may still read the pages being returned
        release_pages_below(kv, kv->hi);
        cudaFree(kv->d_table);
    }
    P->n_seqs--;
    const bool owns = kv->owns_pool;
    delete kv;
    if (owns) pool_free(P);
    return 0;
}

int bebelm_kv_clone(const bebelm_kv* src, bebelm_kv** dst) {
    TRY(validate_kv(src));
    if (!dst) return fail(BEBELM_ERR_INVALID, "dst is null");
    *dst = nullptr;
    bebelm_kv_pool* SP = src->pool;
    DeviceGuard g(SP->device);
    bebelm_kv* kv = nullptr;
    if (src->owns_pool) {
        TRY(bebelm_kv_create(SP->n_layers, SP->n_kv, kHeadDim, src->max_context, kPageTokens, SP->dtype, SP->device,
                             &kv));
    } else {
        TRY(seq_create(SP, src->max_context, false, &kv));
    }
    bebelm_kv_pool* DP = kv->pool;
    const long long n = src->hi - src->lo;
    if ((size_t)n > DP->free_list.size()) {
        bebelm_kv_destroy(kv);
        return fail(BEBELM_ERR_OOM, "page pool exhausted while cloning (%lld pages needed)", n);
    }
    kv->lo = src->lo;
    kv->hi = src->hi;
    kv->base = src->base;
    kv->len = src->len;
    kv->pos = src->pos;
    const size_t page_bytes = SP->page_bytes;
    for (long long L = src->lo; L < src->hi; ++L) {
        const int phys = DP->free_list.back();
        DP->free_list.pop_back();
        kv->table[L % kv->cap] = phys;
        const int sp = src->table[L % src->cap];
        cudaError_t e = cudaMemcpyAsync(DP->mem + (size_t)phys * DP->page_bytes, SP->mem + (size_t)sp * SP->page_bytes,
                                        page_bytes, cudaMemcpyDeviceToDevice, 0);
        if (e != cudaSuccess) {
            bebelm_kv_destroy(kv);
            return fail(BEBELM_ERR_CUDA, "clone copy failed: %s", cudaGetErrorString(e));
        }
    }
    int rc = upload_table(kv, kv->lo, kv->hi, 0);
    if (rc == 0 && cudaDeviceSynchronize() != cudaSuccess) rc = fail(BEBELM_ERR_CUDA, "clone sync failed");
    if (rc) {
        bebelm_kv_destroy(kv);
        return rc;
    }
    *dst = kv;
    return 0;
}

int bebelm_kv_clear(bebelm_kv* kv) {
    TRY(validate_kv(kv));
    DeviceGuard g(kv->pool->device);
    cudaDeviceSynchronize();
    release_pages_below(kv, kv->hi);
    kv->lo = kv->hi = 0;
    std::fill(kv->base.begin(), kv->base.end(), 0);
    std::fill(kv->len.begin(), kv->len.end(), 0);
    kv->pos = 0;
    return 0;
}

int bebelm_kv_len(const bebelm_kv* kv, size_t* out) {
    TRY(validate_kv(kv));
    if (!out) return fail(BEBELM_ERR_INVALID, "out is null");
    long long m = 0;
    for (long long l : kv->len) m = std::max(m, l);
    *out = (size_t)m;
    return 0;
}

int bebelm_kv_layer_len(const bebelm_kv* kv, int layer, size_t* out) {
    TRY(validate_layer(kv, layer));
    if (!out) return fail(BEBELM_ERR_INVALID, "out is null");
    *out = (size_t)kv->len[layer];
    return 0;
}

int bebelm_kv_pos(const bebelm_kv* kv, size_t* out) {
    TRY(validate_kv(kv));
    if (!out) return fail(BEBELM_ERR_INVALID, "out is null");
    *out = kv->pos;
    return 0;
}

int bebelm_kv_set_pos(bebelm_kv* kv, size_t pos) {
    TRY(validate_kv(kv));
    kv->pos = pos;
    return 0;
}

int bebelm_kv_evict_front(bebelm_kv* kv, size_t n) {
    TRY(validate_kv(kv));
    for (size_t l = 0; l < kv->len.size(); ++l) {
        if (kv->len[l] >= (long long)n) {  // layers shorter than n are left alone (src/cache.rs:43)
            kv->base[l] += (long long)n;
            kv->len[l] -= (long long)n;
        }
    }
    recompute_lo(kv);
    return 0;
}

int bebelm_kv_append(bebelm_kv* kv, int layer, const float* k, const float* v, size_t t, int mem, void* stream) {
    TRY(validate_layer(kv, layer));
    TRY(check_mem(mem));
    if (t == 0) return 0;
    if (!k || !v) return fail(BEBELM_ERR_INVALID, "k and v must be non-null");
    bebelm_kv_pool* P = kv->pool;
    DeviceGuard g(P->device);
    cudaStream_t s = as_stream(stream);
    const size_t row = (size_t)P->n_kv * kHeadDim;
    const float *dk = k, *dv = v;
    if (mem == BEBELM_MEM_HOST) {
        void *pk = nullptr, *pv = nullptr;
        Stage st[2] = {{k, sizeof(float) * row * t, &pk}, {v, sizeof(float) * row * t, &pv}};
        TRY(stage_in(P, st, 2, 0, nullptr, s));
        dk = static_cast<const float*>(pk);
        dv = static_cast<const float*>(pv);
    }
    long long slot0 = 0;
    TRY(reserve(kv, layer, t, &slot0, s));
    NormRopeArgs a{};
    a.k = dk;
    a.v = dv;
    a.T = (int)t;
    a.n_heads = 0;
    a.n_kv = P->n_kv;
    a.head_dim = kHeadDim;
    a.norm_k = 0;
    a.append = 1;
    a.pv = P->view(layer);
    a.table = kv->d_table;
    a.cap = kv->cap;
    a.slot0 = slot0;
    CUDA_TRY(launch_norm_rope(a, s));
    P->last_writes.assign(1, {kv, layer, slot0});
    if (mem == BEBELM_MEM_HOST) CUDA_TRY(cudaStreamSynchronize(s));
    return 0;
}

int bebelm_kv_read(const bebelm_kv* kv, int layer, float* k_out, float* v_out, int mem, void* stream) {
    TRY(validate_layer(kv, layer));
    TRY(check_mem(mem));
    bebelm_kv_pool* P = kv->pool;
    DeviceGuard g(P->device);
    cudaStream_t s = as_stream(stream);
    const long long len = kv->len[layer];
    const size_t bytes = sizeof(float) * (size_t)len * P->n_kv * kHeadDim;
    if (len == 0) return 0;
    if (mem == BEBELM_MEM_DEVICE) {
        CUDA_TRY(launch_kv_gather(P->view(layer), kv->d_table, kv->cap, kv->base[layer], len, P->n_kv, k_out, v_out, s));
        return 0;
    }
    void* dout = nullptr;
    TRY(stage_in(P, nullptr, 0, 2 * bytes, &dout, s));
    float* dk = static_cast<float*>(dout);
    float* dv = dk + bytes / sizeof(float);
    CUDA_TRY(launch_kv_gather(P->view(layer), kv->d_table, kv->cap, kv->base[layer], len, P->n_kv,
                              k_out ? dk : nullptr, v_out ? dv : nullptr, s));
    // stage_out copies one contiguous block: K then V
    std::vector<float> both;
    both.resize(2 * bytes / sizeof(float));
    TRY(stage_out(P, dout, both.data(), 2 * bytes, s));
    if (k_out) std::memcpy(k_out, both.data(), bytes);
    if (v_out) std::memcpy(v_out, both.data() + bytes / sizeof(float), bytes);
    return 0;
}

}  // extern "C"

extern "C" {

int bebelm_norm_rope_heads(float* buf, size_t n_tokens, int n_heads, int head_dim, const float* gain, size_t pos0,
                           float theta, float eps, int mem, void* stream) {
    TRY(check_mem(mem));
    if (!buf || !gain) return fail(BEBELM_ERR_INVALID, "buf and gain must be non-null");
    if (n_heads <= 0 || head_dim <= 0 || head_dim > 64 || head_dim % 2)
        return fail(BEBELM_ERR_UNSUPPORTED, "head_dim must be even and in [2, 64] (got %d), n_heads > 0", head_dim);
    if (n_tokens == 0) return 0;
    int dev;
    TRY(current_device(&dev));
    cudaStream_t s = as_stream(stream);
    const size_t n = n_tokens * (size_t)n_heads * head_dim;
    NormRopeArgs a{};
    a.T = (int)n_tokens;
    a.n_heads = n_heads;
    a.n_kv = 0;
    a.head_dim = head_dim;
    a.pos0 = (long long)pos0;
    a.theta_scale = theta_scale_of(theta, head_dim);
    a.eps = eps;
    a.norm_q = 1;
    if (mem == BEBELM_MEM_DEVICE) {
        a.q = buf;
        a.q_gain = gain;
        a.q_out = buf;
        CUDA_TRY(launch_norm_rope(a, s));
        return 0;
    }
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    bebelm_kv_pool* P = nullptr;
    TRY(scratch_pool(dev, &P));
    void *dq = nullptr, *dg = nullptr, *dout = nullptr;
    Stage st[2] = {{buf, sizeof(float) * n, &dq}, {gain, sizeof(float) * head_dim, &dg}};
    TRY(stage_in(P, st, 2, sizeof(float) * n, &dout, s));
    a.q = static_cast<const float*>(dq);
    a.q_gain = static_cast<const float*>(dg);
    a.q_out = static_cast<float*>(dout);
    CUDA_TRY(launch_norm_rope(a, s));
    return stage_out(P, dout, buf, sizeof(float) * n, s);
}

int bebelm_attn_decode_host(const float* q, const float* k, const float* v, size_t n_ctx, int n_heads, int n_kv_heads,
                            int head_dim, float* out) {
    TRY(check_geometry(n_heads, n_kv_heads));
    if (head_dim <= 0 || head_dim > 64)
        return fail(BEBELM_ERR_UNSUPPORTED, "head_dim must be in [1, 64] (got %d)", head_dim);
    if (!q || !out || (n_ctx && (!k || !v))) return fail(BEBELM_ERR_INVALID, "null buffer");
    const size_t hidden = (size_t)n_heads * head_dim;
    if (n_ctx == 0) {  // softmax of nothing: the reference leaves zeros
        std::memset(out, 0, sizeof(float) * hidden);
        return 0;
    }
    int dev;
    TRY(current_device(&dev));
    // re-lay out to head_dim 64 (zero padding changes no dot product and no output column)
    std::vector<float> qp((size_t)n_heads * 64, 0.f), kp, vp;
    const float *kk = k, *vv = v, *qq = q;
    if (head_dim != 64) {
        kp.assign(n_ctx * n_kv_heads * 64, 0.f);
        vp.assign(n_ctx * n_kv_heads * 64, 0.f);
        for (size_t r = 0; r < n_ctx * (size_t)n_kv_heads; ++r) {
            std::memcpy(&kp[r * 64], k + r * head_dim, sizeof(float) * head_dim);
            std::memcpy(&vp[r * 64], v + r * head_dim, sizeof(float) * head_dim);
        }
        for (int h = 0; h < n_heads; ++h) std::memcpy(&qp[(size_t)h * 64], q + (size_t)h * head_dim, sizeof(float) * head_dim);
        kk = kp.data();
        vv = vp.data();
        qq = qp.data();
    }
    bebelm_kv* kv = nullptr;
    TRY(bebelm_kv_create(1, n_kv_heads, 64, n_ctx, kPageTokens, BEBELM_F32, dev, &kv));
    int rc = bebelm_kv_append(kv, 0, kk, vv, n_ctx, BEBELM_MEM_HOST, nullptr);
    if (rc == 0) {
        bebelm_kv_pool* P = kv->pool;
        void *dq = nullptr, *dout = nullptr;
        Stage st[1] = {{qq, sizeof(float) * n_heads * 64, &dq}};
        rc = stage_in(P, st, 1, sizeof(float) * n_heads * 64, &dout, 0);
        if (rc == 0) {
            std::vector<Window> w{{kv, kv->base[0], kv->len[0], -1, 0}};
            rc = run_decode(P, w, 0, n_heads, static_cast<const float*>(dq), static_cast<float*>(dout),
                            1.0f / sqrtf((float)head_dim), nullptr, 0);
        }
        if (rc == 0) rc = stage_out(P, dout, qp.data(), sizeof(float) * n_heads * 64, 0);
        if (rc == 0)
            for (int h = 0; h < n_heads; ++h)
                std::memcpy(out + (size_t)h * head_dim, &qp[(size_t)h * 64], sizeof(float) * head_dim);
    }
    bebelm_kv_destroy(kv);
    return rc;
}

int bebelm_attn_step(bebelm_kv* kv, int layer, int n_heads, const float* q, const float* k, const float* v,
                     const float* q_gain, const float* k_gain, float theta, float eps, size_t pos, float* out, int mem,
                     void* stream) {
    TRY(validate_layer(kv, layer));
    TRY(check_mem(mem));
    bebelm_kv_pool* P = kv->pool;
    TRY(check_geometry(n_heads, P->n_kv));
    if (!q || !k || !v || !q_gain || !k_gain || !out) return fail(BEBELM_ERR_INVALID, "null buffer");
    DeviceGuard g(P->device);
    cudaStream_t s = as_stream(stream);
    const size_t qn = (size_t)n_heads * kHeadDim, kvn = (size_t)P->n_kv * kHeadDim;
    const float *dq = q, *dk = k, *dv = v, *dqg = q_gain, *dkg = k_gain;
    float* dout = out;
    if (mem == BEBELM_MEM_HOST) {
        void *a0, *a1, *a2, *a3, *a4, *o;
        Stage st[5] = {{q, 4 * qn, &a0}, {k, 4 * kvn, &a1}, {v, 4 * kvn, &a2}, {q_gain, 4 * 64, &a3}, {k_gain, 4 * 64, &a4}};
        TRY(stage_in(P, st, 5, 4 * qn, &o, s));
        dq = (const float*)a0; dk = (const float*)a1; dv = (const float*)a2;
        dqg = (const float*)a3; dkg = (const float*)a4; dout = (float*)o;
    }
    long long slot0 = 0;
    TRY(reserve(kv, layer, 1, &slot0, s));
    const FusedStep fs{dq, dk, dv, dqg, dkg, theta_scale_of(theta, kHeadDim), eps};
    std::vector<Window> w{{kv, kv->base[layer], kv->len[layer], slot0, (long long)pos}};
    TRY(run_decode(P, w, layer, n_heads, nullptr, dout, 0.125f, &fs, s));
    if (mem == BEBELM_MEM_HOST) return stage_out(P, dout, out, 4 * qn, s);
    return 0;
}

int bebelm_attn_decode_batched(bebelm_kv* const* seqs, int n_seqs, int layer, int n_heads, const float* q,
                               const float* k, const float* v, const float* q_gain, const float* k_gain, float theta,
                               float eps, const size_t* pos, float* out, int mem, void* stream) {
    TRY(check_mem(mem));
    if (!seqs || n_seqs <= 0 || !pos) return fail(BEBELM_ERR_INVALID, "need n_seqs > 0 sequences and positions");
    bebelm_kv_pool* P = seqs[0] ? seqs[0]->pool : nullptr;
    for (int i = 0; i < n_seqs; ++i) {
        TRY(validate_layer(seqs[i], layer));
        if (seqs[i]->pool != P) return fail(BEBELM_ERR_INVALID, "batched decode needs all sequences in one pool");
        for (int j = 0; j < i; ++j)
            if (seqs[j] == seqs[i]) return fail(BEBELM_ERR_INVALID, "sequence %d appears twice", i);
    }
    TRY(check_geometry(n_heads, P->n_kv));
    if (!q || !k || !v || !q_gain || !k_gain || !out) return fail(BEBELM_ERR_INVALID, "null buffer");
    DeviceGuard g(P->device);
    cudaStream_t s = as_stream(stream);
    const size_t qn = (size_t)n_heads * kHeadDim * n_seqs, kvn = (size_t)P->n_kv * kHeadDim * n_seqs;
    const float *dq = q, *dk = k, *dv = v, *dqg = q_gain, *dkg = k_gain;
    float* dout = out;
    if (mem == BEBELM_MEM_HOST) {
        void *a0, *a1, *a2, *a3, *a4, *o;
        Stage st[5] = {{q, 4 * qn, &a0}, {k, 4 * kvn, &a1}, {v, 4 * kvn, &a2}, {q_gain, 4 * 64, &a3}, {k_gain, 4 * 64, &a4}};
        TRY(stage_in(P, st, 5, 4 * qn, &o, s));
        dq = (const float*)a0; dk = (const float*)a1; dv = (const float*)a2;
        dqg = (const float*)a3; dkg = (const float*)a4; dout = (float*)o;
    }
    // capacity first for every sequence, so a failure leaves no window changed
    for (int i = 0; i < n_seqs; ++i) {
        const bebelm_kv* kv = seqs[i];
        long long b = kv->base[layer], n = kv->len[layer];
        if (n == 0 && b < kv->lo * kPageTokens) b = kv->lo * kPageTokens;
        if ((b + n + 1 + kPageTokens - 1) / kPageTokens - kv->lo > kv->cap)
            return fail(BEBELM_ERR_CAPACITY, "sequence %d is full: evict_front first", i);
    }
    std::vector<Window> w(n_seqs);
    for (int i = 0; i < n_seqs; ++i) {
        long long slot = 0;
        TRY(reserve(seqs[i], layer, 1, &slot, s));
        w[i] = {seqs[i], seqs[i]->base[layer], seqs[i]->len[layer], slot, (long long)pos[i]};
    }
    const FusedStep fs{dq, dk, dv, dqg, dkg, theta_scale_of(theta, kHeadDim), eps};
    TRY(run_decode(P, w, layer, n_heads, nullptr, dout, 0.125f, &fs, s));
    if (mem == BEBELM_MEM_HOST) return stage_out(P, dout, out, 4 * qn, s);
    return 0;
}

}  // extern "C"

namespace {

// Device part of a chunked prefill (src/model.rs:232-254 middle section): t tokens' q/k/v
// (fp32, or bf16 when in_bf16) are normed, roped and appended, then attend causally to the
// window. tc: the tensor-core kernel (bf16 operands; the inputs are rounded to bf16 by the
// norm kernel when they are fp32), else the exact fp32 split-K path with one causal window
// per token. dout [t][n_heads*64] fp32 on the device.
// A rank's share of a KV-head-sharded prefill: which heads of the replicated full input rows
// are this call's, and where the gathered output goes (the landing zones of a peer group).
struct PrefillShard {
    int q_row_heads, q_head0, kv_row_heads, kv_head0;
    unsigned long long* const* bufs;
    const unsigned long long* epoch;
    int world, rank;
    size_t slice;
};

int prefill_device(bebelm_kv* kv, int layer, int n_heads, const void* dq, const void* dk, const void* dv, bool in_bf16,
                   bool tc, size_t t, size_t pos0, const float* dqg, const float* dkg, float theta, float eps,
                   float* dout, cudaStream_t s, const PrefillShard* shard = nullptr) {
    bebelm_kv_pool* P = kv->pool;
    const size_t qn = (size_t)n_heads * kHeadDim * t;
    long long slot0 = 0;
    TRY(reserve(kv, layer, t, &slot0, s));
    const long long len_before = kv->len[layer] - (long long)t;
    if (tc) {
        // tensor-core path: bf16 q and the bf16 window [prefix | new keys] feed kernel 2
        const size_t kvrow = (size_t)P->n_kv * kHeadDim;
        const size_t s_total = (size_t)len_before + t;
        TRY(P->pf.ensure(2 * (qn + 2 * s_total * kvrow) + 1024, false, s));
        __nv_bfloat16* qb = P->pf.as<__nv_bfloat16>();
        __nv_bfloat16* kb = qb + ((qn + 127) & ~size_t(127));
        __nv_bfloat16* vb = kb + ((s_total * kvrow + 127) & ~size_t(127));
        // descriptors first, so the two kernels below go out back to back
        PrefillArgs pa{};
        pa.q = qb; pa.k = kb; pa.v = vb; pa.out = dout;
        pa.t = (int)t; pa.len_before = (int)len_before; pa.n_heads = n_heads; pa.n_kv = P->n_kv;
        pa.scale_log2 = 0.125f * 1.4426950408889634f;
        pa.err = P->err.d;
        if (shard) {
            pa.peer_bufs = shard->bufs;
            pa.peer_epoch = shard->epoch;
            pa.peer_world = shard->world;
            pa.peer_rank = shard->rank;
            pa.peer_slice = shard->slice;
        }
        PrefillMaps maps;
        if (!prefill_make_maps(pa, &maps)) return fail(BEBELM_ERR_CUDA, "building the TMA tensor maps for prefill failed");
        if (len_before > 0)
            CUDA_TRY(launch_kv_gather_bf16(P->view(layer), kv->d_table, kv->cap, kv->base[layer], len_before, P->n_kv,
                                           kb, vb, s));
        NormRopeArgs a{};
        a.q = (const float*)dq; a.k = (const float*)dk; a.v = (const float*)dv; a.q_gain = dqg; a.k_gain = dkg;
        a.T = (int)t; a.n_heads = n_heads; a.n_kv = P->n_kv; a.head_dim = kHeadDim;
        a.pos0 = (long long)pos0;
        a.theta_scale = theta_scale_of(theta, kHeadDim);
        a.eps = eps;
        a.norm_q = 1; a.norm_k = 1;
        a.q_bf16 = qb; a.k_bf16 = kb + (size_t)len_before * kvrow; a.v_bf16 = vb + (size_t)len_before * kvrow;
        a.append = 1; a.pv = P->view(layer); a.table = kv->d_table; a.cap = kv->cap; a.slot0 = slot0;
        a.in_bf16 = in_bf16 ? 1 : 0;  // norm + RoPE read the inputs in their own type
        if (shard) {
            a.q_row_heads = shard->q_row_heads;
            a.q_head0 = shard->q_head0;
            a.kv_row_heads = shard->kv_row_heads;
            a.kv_head0 = shard->kv_head0;
        }
        a.trigger_dependents = 1;  // the prefill kernel sets up while this one runs, then waits for it
        CUDA_TRY(launch_norm_rope(a, s));
        P->last_writes.assign(1, {kv, layer, slot0});
        CUDA_TRY(launch_prefill(pa, maps, s));
        P->last_writes.clear();
        return 0;
    }
    if (in_bf16) return fail(BEBELM_ERR_UNSUPPORTED, "bf16 inputs take the tensor-core path");
    if (shard) return fail(BEBELM_ERR_UNSUPPORTED, "a gathered prefill takes the tensor-core path");
    TRY(P->qn.ensure(4 * qn, false, s));
    NormRopeArgs a{};
    a.q = (const float*)dq; a.k = (const float*)dk; a.v = (const float*)dv; a.q_gain = dqg; a.k_gain = dkg;
    a.T = (int)t; a.n_heads = n_heads; a.n_kv = P->n_kv; a.head_dim = kHeadDim;
    a.pos0 = (long long)pos0;
    a.theta_scale = theta_scale_of(theta, kHeadDim);
    a.eps = eps;
    a.norm_q = 1; a.norm_k = 1;
    a.q_out = P->qn.as<float>();
    a.append = 1; a.pv = P->view(layer); a.table = kv->d_table; a.cap = kv->cap; a.slot0 = slot0;
    CUDA_TRY(launch_norm_rope(a, s));
    P->last_writes.assign(1, {kv, layer, slot0});
    // token i sees the window up to and including itself (src/model.rs:240-244)
    std::vector<Window> w(t);
    for (size_t i = 0; i < t; ++i) w[i] = {kv, kv->base[layer], len_before + (long long)i + 1, -1, 0};
    TRY(run_decode(P, w, layer, n_heads, P->qn.as<float>(), dout, 0.125f, nullptr, s));
    return 0;
}

}  // namespace

extern "C" {

int bebelm_attn_prefill(bebelm_kv* kv, int layer, int n_heads, const void* q, const void* k, const void* v,
                        int in_dtype, size_t t, size_t pos0, const float* q_gain, const float* k_gain, float theta,
                        float eps, float* out, int mem, void* stream) {
    TRY(validate_layer(kv, layer));
    TRY(check_mem(mem));
    bebelm_kv_pool* P = kv->pool;
    TRY(check_geometry(n_heads, P->n_kv));
    if (in_dtype != BEBELM_F32 && in_dtype != BEBELM_BF16 && in_dtype != BEBELM_F32_TENSOR)
        return fail(BEBELM_ERR_UNSUPPORTED, "in_dtype must be BEBELM_F32, BEBELM_BF16 or BEBELM_F32_TENSOR");
    if (t == 0) return 0;
    if (!q || !k || !v || !q_gain || !k_gain || !out) return fail(BEBELM_ERR_INVALID, "null buffer");
    if (t > (size_t)INT32_MAX / (size_t)n_heads) return fail(BEBELM_ERR_INVALID, "t too large");
    DeviceGuard g(P->device);
    cudaStream_t s = as_stream(stream);
    const size_t esz = in_dtype == BEBELM_BF16 ? 2 : 4;
    const size_t qn = (size_t)n_heads * kHeadDim * t, kvn = (size_t)P->n_kv * kHeadDim * t;
    const void *dq = q, *dk = k, *dv = v;
    const float *dqg = q_gain, *dkg = k_gain;
    float* dout = out;
    if (mem == BEBELM_MEM_HOST) {
        void *a0, *a1, *a2, *a3, *a4, *o;
        Stage st[5] = {{q, esz * qn, &a0}, {k, esz * kvn, &a1}, {v, esz * kvn, &a2}, {q_gain, 4 * 64, &a3}, {k_gain, 4 * 64, &a4}};
        TRY(stage_in(P, st, 5, 4 * qn, &o, s));
        dq = a0; dk = a1; dv = a2;
        dqg = (const float*)a3; dkg = (const float*)a4; dout = (float*)o;
    }
    const bool bf = in_dtype == BEBELM_BF16, tc = in_dtype != BEBELM_F32;
    TRY(prefill_device(kv, layer, n_heads, dq, dk, dv, bf, tc, t, pos0, dqg, dkg, theta, eps, dout, s));
    if (mem == BEBELM_MEM_HOST) return stage_out(P, dout, out, 4 * qn, s);
    return 0;
}

}  // extern "C"

extern "C" {

int bebelm_attn_decode_cached(const bebelm_kv* kv, int layer, int n_heads, const float* q, float* out, int mem,
                              void* stream) {
    TRY(validate_layer(kv, layer));
    TRY(check_mem(mem));
    bebelm_kv_pool* P = kv->pool;
    TRY(check_geometry(n_heads, P->n_kv));
    if (!q || !out) return fail(BEBELM_ERR_INVALID, "null buffer");
    DeviceGuard g(P->device);
    cudaStream_t s = as_stream(stream);
    const size_t qn = (size_t)n_heads * kHeadDim;
    const float* dq = q;
    float* dout = out;
    if (mem == BEBELM_MEM_HOST) {
        void *a0, *o;
        Stage st[1] = {{q, 4 * qn, &a0}};
        TRY(stage_in(P, st, 1, 4 * qn, &o, s));
        dq = (const float*)a0;
        dout = (float*)o;
    }
    if (kv->len[layer] == 0) {
        CUDA_TRY(cudaMemsetAsync(dout, 0, 4 * qn, s));
    } else {
        std::vector<Window> w{{kv, kv->base[layer], kv->len[layer], -1, 0}};
        TRY(run_decode(P, w, layer, n_heads, dq, dout, 0.125f, nullptr, s));
    }
    if (mem == BEBELM_MEM_HOST) return stage_out(P, dout, out, 4 * qn, s);
    return 0;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Decode without any allocation at call time.
//
// bebelm_attn_decode_cached keeps its split partials and counters in pool scratch
// that grows on demand with cudaMalloc. This variant takes them from a fixed
// file-scope device array instead, for callers that must not allocate device
// memory while they run (see the header). The array is process-wide: every GPU
// that loads this library holds kNoAllocScratchFloats floats of it until exit,
// and every call on a device shares it.
namespace {

constexpr size_t kNoAllocScratchFloats = (size_t)1 << 19;  // 2 MiB of split partials and counters
constexpr size_t kNoAllocCounterWords = 1024;              // tail of the array: split counters
constexpr size_t kNoAllocPartialFloats = kNoAllocScratchFloats - kNoAllocCounterWords - 64;

static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];

std::mutex g_noalloc_mu;
float* g_noalloc_addr[64] = {};  // device address of g_noalloc_scratch, per device

// Once per device, with that device current: look up the array's device address (the
// host-side symbol is only a stand-in) and zero the counters and error word.
int noalloc_scratch(int dev, cudaStream_t s, float** out) {
    if (dev < 0 || dev >= 64) return fail(BEBELM_ERR_INVALID, "device %d unsupported", dev);
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_addr[dev]) {
        float* ptr = nullptr;
        cudaError_t e = cudaGetSymbolAddress((void**)&ptr, g_noalloc_scratch);
        if (e != cudaSuccess || !ptr)
            return fail(BEBELM_ERR_CUDA, "cudaGetSymbolAddress of the no-allocation scratch failed: %s",
                        cudaGetErrorString(e));
        e = cudaMemsetAsync(ptr + kNoAllocPartialFloats, 0, sizeof(float) * (kNoAllocCounterWords + 64), s);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) return fail(BEBELM_ERR_CUDA, "clearing the no-allocation scratch failed: %s", cudaGetErrorString(e));
        g_noalloc_addr[dev] = ptr;
    }
    *out = g_noalloc_addr[dev];
    return 0;
}

void clear_noalloc_counters(int dev, cudaStream_t s) {
    if (dev < 0 || dev >= 64) return;
    float* ptr = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_noalloc_mu);
        ptr = g_noalloc_addr[dev];
    }
    if (ptr) cudaMemsetAsync(ptr + kNoAllocPartialFloats, 0, sizeof(unsigned) * kNoAllocCounterWords, s);
}

}  // namespace

namespace bebelm {
int g_expire_waits = 0;
}

extern "C" int bebelm_debug_expire_next_wait(int n_launches) {
    if (n_launches < 0) return fail(BEBELM_ERR_INVALID, "n_launches < 0");
    g_expire_waits = n_launches;
    return 0;
}

extern "C" int bebelm_attn_decode_cached_noalloc(const bebelm_kv* kv, int layer, int n_heads, const float* q,
                                                 float* out, void* stream) {
    TRY(validate_layer(kv, layer));
    bebelm_kv_pool* P = kv->pool;
    TRY(check_geometry(n_heads, P->n_kv));
    if (!q || !out) return fail(BEBELM_ERR_INVALID, "null buffer");
    DeviceGuard g(P->device);
    cudaStream_t s = as_stream(stream);
    float* scratch = nullptr;
    TRY(noalloc_scratch(P->device, s, &scratch));
    const long long len = kv->len[layer], base = kv->base[layer];
    if (len == 0) {
        CUDA_TRY(cudaMemsetAsync(out, 0, sizeof(float) * (size_t)n_heads * kHeadDim, s));
        return 0;
    }
    // the same split plan as run_decode for one window
    const int group = n_heads / P->n_kv;
    int hpc, n_sub;
    pick_heads_per_cta(group, &hpc, &n_sub);
    const int NY = P->n_kv * n_sub;
    const long long npages = (base + len - 1) / kPageTokens - base / kPageTokens + 1;
    const long long target = (long long)P->num_sms * 2;
    long long per = std::max<long long>(1, (npages * NY + target - 1) / target);
    per = std::min<long long>(per, kDecodeMaxPagesPerSplit);
    const long long n_splits = (npages + per - 1) / per;
    const size_t need = (size_t)n_splits * NY * hpc * (kHeadDim + 2);
    if ((size_t)NY > kNoAllocCounterWords)
        return fail(BEBELM_ERR_INVALID,
                    "%d kv heads x %d head groups need %d split counters; the no-allocation path holds at most %zu",
                    P->n_kv, n_sub, NY, kNoAllocCounterWords);
    if (need > kNoAllocPartialFloats)
        return fail(BEBELM_ERR_INVALID,
                    "window of %lld positions needs %zu scratch floats (%lld splits x %d heads); the no-allocation "
                    "path holds at most %zu",
                    len, need, n_splits, NY * hpc, kNoAllocPartialFloats);
    DecodeArgs a{};
    a.one.table = kv->d_table;
    a.one.cap = kv->cap;
    a.one.len = (int)len;
    a.one.base = base;
    a.one.split0 = 0;
    a.one.n_splits = (int)n_splits;
    a.one.new_slot = -1;
    a.one.pos = 0;
    a.one.dep_slot = dep_slot_for(P, kv, layer);
    a.n_seqs = 1;
    a.pv = P->view(layer);
    a.q = q;
    a.out = out;
    a.part_acc = scratch;
    a.part_ml = scratch + (size_t)n_splits * NY * hpc * kHeadDim;
    a.counters = reinterpret_cast<unsigned*>(scratch + kNoAllocPartialFloats);
    a.err = P->err.d;  // the pool's mapped error word (allocated with the pool): bebelm_kv_check reads it
    a.n_heads = n_heads;
    a.n_kv = P->n_kv;
    a.group = group;
    a.hpc = hpc;
    a.n_sub = n_sub;
    a.pages_per_split = (int)per;
    a.total_splits = (int)n_splits;
    a.scale_log2 = 0.125f * 1.4426950408889634f;
    a.pdl = 1;
    if (g_expire_waits > 0) {  // test hook (bebelm_debug_expire_next_wait)
        a.expire_wait = 1;
        --g_expire_waits;
    }
    CUDA_TRY(launch_decode(a, s));
    record_decode_out(s, out, (size_t)n_heads * kHeadDim * 4);
    return 0;
}

// ---------------------------------------------------------------------------
// Fused KV-head-sharded steps: decode (or prefill) + all-gather over peer memory (NVLink stores).
//
// Each rank owns a landing zone allocated with cudaMalloc and exported by CUDA IPC:
//   [256-byte header, unused][parity 0: world x slice words][parity 1: world x slice words]
// A word is 8 bytes: the step's tag (low 32 bits of its epoch) above a float's bits. Step e
// writes parity e&1 of every rank's zone with plain stores; a rank's gather kernel polls its own
// zone until every word carries tag e, copies the floats out and advances the epoch (a device
// word, so a captured graph of steps replays unchanged). A rank may run one step ahead of a peer
// that is still copying out: a writer of step e+2 has seen every rank's step e+1 words, which a
// rank writes only after (stream order) its own copy-out of step e.
// ---------------------------------------------------------------------------
constexpr int kMaxPeers = 32;  // flags fit the 256-byte header

struct bebelm_peer_group {
    int device = -1, world = 0, rank = 0;
    size_t slice = 0;  // floats per rank per parity
    char* zone = nullptr;
    char* peer_base[kMaxPeers] = {};  // opened IPC mappings (own entry: zone)
    DevBuf tables;                    // u64* bufs[world], the epoch word, the gather's done counter
    bool connected = false;
    size_t zone_bytes() const { return 256 + 2 * (size_t)world * slice * sizeof(unsigned long long); }
    unsigned long long* const* d_bufs() const { return tables.as<unsigned long long* const>(); }
    // Steps completed on this rank, in device memory: a step is epoch + 1; its gather kernel
    // stores that back once the gathered output is copied out. Keeping it on the device lets a
    // captured graph of steps replay without any launch argument changing.
    unsigned long long* d_epoch() const {
        return reinterpret_cast<unsigned long long*>(tables.as<char>() + sizeof(void*) * world);
    }
    unsigned* d_done() const { return reinterpret_cast<unsigned*>(d_epoch() + 1); }
    const unsigned long long* local_zone() const { return reinterpret_cast<const unsigned long long*>(zone + 256); }
};

namespace {

// The gather kernel that follows a decode step whose CTAs store into the landing zones: it
// waits for every rank's words of this step and copies the gathered [world][slice] out.
int peer_gather_out(const bebelm_peer_group* g, bebelm_kv_pool* P, float* dout, cudaStream_t s) {
    CUDA_TRY(launch_gather_ll(g->local_zone(), g->d_epoch(), g->d_done(), g->world, g->slice, 1, g->slice, dout,
                              P->err.d, s));
    return 0;
}

}  // namespace

extern "C" {

int bebelm_kv_check(const bebelm_kv* kv, void* stream) {
    if (!kv) return fail(BEBELM_ERR_INVALID, "null handle");
    bebelm_kv_pool* P = kv->pool;
    DeviceGuard dg(P->device);
    cudaStream_t s = as_stream(stream);
    CUDA_TRY(cudaStreamSynchronize(s));
    const int derr = P->err.read();
    if (derr) {
        P->err.clear();
        if (P->counters.p) cudaMemsetAsync(P->counters.p, 0, P->counters.bytes, s);
        clear_noalloc_counters(P->device, s);
        cudaStreamSynchronize(s);
        return fail(BEBELM_ERR_TIMEOUT, "a device-side wait timed out (code %d); outputs are invalid", derr);
    }
    return 0;
}

int bebelm_peer_group_create(int device, int world, int rank, size_t slice_floats, void* handle_out,
                             bebelm_peer_group** out) {
    if (!out || !handle_out) return fail(BEBELM_ERR_INVALID, "null argument");
    *out = nullptr;
    if (world < 1 || world > kMaxPeers || rank < 0 || rank >= world)
        return fail(BEBELM_ERR_INVALID, "rank %d / world %d out of range (world <= %d)", rank, world, kMaxPeers);
    if (slice_floats == 0 || slice_floats % 64)
        return fail(BEBELM_ERR_INVALID, "slice_floats (%zu) must be a positive multiple of 64", slice_floats);
    int n_dev = 0;
    CUDA_TRY(cudaGetDeviceCount(&n_dev));
    if (device < 0 || device >= n_dev) return fail(BEBELM_ERR_INVALID, "device %d not present", device);
    DeviceGuard dg(device);
    auto* g = new bebelm_peer_group();
    g->device = device;
    g->world = world;
    g->rank = rank;
    g->slice = slice_floats;
    cudaError_t e = cudaMalloc(&g->zone, g->zone_bytes());
    if (e == cudaSuccess) e = cudaMemset(g->zone, 0, g->zone_bytes());
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle_out), g->zone);
    if (e != cudaSuccess) {
        if (g->zone) cudaFree(g->zone);
        delete g;
        return fail(BEBELM_ERR_CUDA, "peer zone: %s", cudaGetErrorString(e));
    }
    g->peer_base[rank] = g->zone;
    *out = g;
    return 0;
}

int bebelm_peer_group_connect(bebelm_peer_group* g, const void* handles) {
    if (!g || !handles) return fail(BEBELM_ERR_INVALID, "null argument");
    if (g->connected) return fail(BEBELM_ERR_INVALID, "peer group already connected");
    DeviceGuard dg(g->device);
    const auto* h = static_cast<const cudaIpcMemHandle_t*>(handles);
    for (int r = 0; r < g->world; ++r) {
        if (r == g->rank) continue;
        void* p = nullptr;
        cudaError_t e = cudaIpcOpenMemHandle(&p, h[r], cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            for (int q = 0; q < r; ++q)
                if (q != g->rank && g->peer_base[q]) cudaIpcCloseMemHandle(g->peer_base[q]), g->peer_base[q] = nullptr;
            return fail(BEBELM_ERR_CUDA, "opening rank %d's zone: %s", r, cudaGetErrorString(e));
        }
        g->peer_base[r] = static_cast<char*>(p);
    }
    std::vector<void*> tab((size_t)g->world);
    for (int r = 0; r < g->world; ++r) tab[r] = g->peer_base[r] + 256;
    TRY(g->tables.ensure(sizeof(void*) * tab.size() + 2 * sizeof(unsigned long long), true));
    CUDA_TRY(cudaMemcpy(g->tables.p, tab.data(), sizeof(void*) * tab.size(), cudaMemcpyHostToDevice));
    CUDA_TRY(cudaDeviceSynchronize());  // the zeroed epoch word too
    g->connected = true;
    return 0;
}

int bebelm_peer_group_destroy(bebelm_peer_group* g) {
    if (!g) return 0;
    DeviceGuard dg(g->device);
    cudaDeviceSynchronize();
    for (int r = 0; r < g->world; ++r)
        if (r != g->rank && g->peer_base[r]) cudaIpcCloseMemHandle(g->peer_base[r]);
    g->tables.release();
    if (g->zone) cudaFree(g->zone);
    delete g;
    return 0;
}

int bebelm_attn_step_allgather(bebelm_kv* kv, bebelm_peer_group* g, int layer, int n_heads, const float* q,
                               const float* k, const float* v, const float* q_gain, const float* k_gain, float theta,
                               float eps, size_t pos, float* out, int mem, void* stream) {
    TRY(validate_layer(kv, layer));
    TRY(check_mem(mem));
    if (!g || !g->connected) return fail(BEBELM_ERR_INVALID, "peer group missing or not connected");
    bebelm_kv_pool* P = kv->pool;
    TRY(check_geometry(n_heads, P->n_kv));
    if (P->device != g->device) return fail(BEBELM_ERR_INVALID, "cache and peer group are on different devices");
    const size_t qn = (size_t)n_heads * kHeadDim, kvn = (size_t)P->n_kv * kHeadDim;
    if (qn != g->slice)
        return fail(BEBELM_ERR_INVALID, "n_heads*64 (%zu) differs from the group's slice (%zu)", qn, g->slice);
    if (!q || !k || !v || !q_gain || !k_gain || !out) return fail(BEBELM_ERR_INVALID, "null buffer");
    DeviceGuard dg(P->device);
    cudaStream_t s = as_stream(stream);
    const size_t full = (size_t)g->world * qn;
    const float *dq = q, *dk = k, *dv = v, *dqg = q_gain, *dkg = k_gain;
    float* dout = out;
    if (mem == BEBELM_MEM_HOST) {
        void *a0, *a1, *a2, *a3, *a4, *o;
        Stage st[5] = {{q, 4 * qn, &a0}, {k, 4 * kvn, &a1}, {v, 4 * kvn, &a2}, {q_gain, 4 * 64, &a3}, {k_gain, 4 * 64, &a4}};
        TRY(stage_in(P, st, 5, 4 * full, &o, s));
        dq = (const float*)a0; dk = (const float*)a1; dv = (const float*)a2;
        dqg = (const float*)a3; dkg = (const float*)a4; dout = (float*)o;
    }
    long long slot0 = 0;
    TRY(reserve(kv, layer, 1, &slot0, s));
    const FusedStep fs{dq, dk, dv, dqg, dkg, theta_scale_of(theta, kHeadDim), eps};
    std::vector<Window> w{{kv, kv->base[layer], kv->len[layer], slot0, (long long)pos}};
    const PeerTarget pt{g->d_bufs(), g->world, g->rank, g->d_epoch()};
    TRY(run_decode(P, w, layer, n_heads, nullptr, dout, 0.125f, &fs, s, &pt));
    TRY(peer_gather_out(g, P, dout, s));
    if (mem == BEBELM_MEM_HOST) return stage_out(P, dout, out, 4 * full, s);
    return 0;
}

int bebelm_attn_prefill_allgather(bebelm_kv* kv, bebelm_peer_group* g, int layer, int n_heads, const void* q,
                                  const void* k, const void* v, int in_dtype, size_t t, size_t pos0,
                                  const float* q_gain, const float* k_gain, float theta, float eps, float* out,
                                  void* stream) {
    TRY(validate_layer(kv, layer));
    if (!g || !g->connected) return fail(BEBELM_ERR_INVALID, "peer group missing or not connected");
    bebelm_kv_pool* P = kv->pool;
    TRY(check_geometry(n_heads, P->n_kv));
    if (P->device != g->device) return fail(BEBELM_ERR_INVALID, "cache and peer group are on different devices");
    if (in_dtype != BEBELM_BF16 && in_dtype != BEBELM_F32_TENSOR)
        return fail(BEBELM_ERR_UNSUPPORTED, "a gathered prefill takes BEBELM_BF16 or BEBELM_F32_TENSOR inputs");
    if (t == 0) return 0;
    if (!q || !k || !v || !q_gain || !k_gain || !out) return fail(BEBELM_ERR_INVALID, "null buffer");
    const size_t row = (size_t)n_heads * kHeadDim;
    if (t * row > g->slice)
        return fail(BEBELM_ERR_CAPACITY, "%zu tokens x %d heads exceed the group's landing zone (%zu floats a rank)", t,
                    n_heads, g->slice);
    DeviceGuard dg(P->device);
    cudaStream_t s = as_stream(stream);
    const PrefillShard sh{n_heads * g->world, n_heads * g->rank, P->n_kv * g->world, P->n_kv * g->rank,
                          g->d_bufs(), g->d_epoch(), g->world, g->rank, g->slice};
    TRY(prefill_device(kv, layer, n_heads, q, k, v, in_dtype == BEBELM_BF16, true, t, pos0, q_gain, k_gain, theta,
                       eps, nullptr, s, &sh));
    CUDA_TRY(launch_gather_ll(g->local_zone(), g->d_epoch(), g->d_done(), g->world, g->slice, t, row, out, P->err.d,
                              s));
    return 0;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Step plans: device-driven decode steps for CUDA-graph capture.
//
// A plan fixes everything a decode step's launch needs except the window, which the kernel
// derives from a step counter in device memory (StepState) and the plan's starting point:
// step n appends slot slot0 + n at position pos0 + n and attends to the last
// min(len0 + n + 1, window) slots. Creating a plan assigns a physical page to every entry
// of the sequence's page ring, so no later step needs the host: the window (at most
// ceil(window/64) + 1 pages) always fits the ring (ceil(max_context/64) + 2 entries). The
// split plan and the grid are sized for the largest window; CTAs past the current window
// contribute empty partials. Finishing folds the steps taken back into the host state.
// ---------------------------------------------------------------------------
struct bebelm_step_plan {
    bebelm_kv* kv = nullptr;
    int layer = 0, n_heads = 0;
    long long slot0 = 0, pos0 = 0, len0 = 0, window = 0;
    int n_splits = 0, per = 0, hpc = 0, n_sub = 0;
    DevBuf state, part, counters;  // StepState, split partials, combine counters
    // whole-operator plans: the layer's weights and the scratch of its projections
    const bebelm_attn_weights* W = nullptr;
    DevBuf lbuf;  // q, k, v, attention output (f32), then Q8 activations (quants, scales, sums)
};

extern "C" {

int bebelm_step_plan_create(bebelm_kv* kv, int layer, int n_heads, size_t window, bebelm_step_plan** out) {
    if (!out) return fail(BEBELM_ERR_INVALID, "out is null");
    *out = nullptr;
    if (!kv || !kv->pool) return fail(BEBELM_ERR_INVALID, "null cache handle");
    if (layer < 0 || layer >= kv->pool->n_layers)
        return fail(BEBELM_ERR_INVALID, "layer %d out of range [0,%d)", layer, kv->pool->n_layers);
    bebelm_kv_pool* P = kv->pool;
    TRY(check_geometry(n_heads, P->n_kv));
    if (window == 0) window = kv->max_context;
    if (window > kv->max_context)
        return fail(BEBELM_ERR_INVALID, "window %zu exceeds the cache's max_context %zu", window, kv->max_context);
    if (kv->len[layer] > (long long)window)
        return fail(BEBELM_ERR_INVALID, "layer %d holds %lld positions, more than the window %zu", layer,
                    kv->len[layer], window);
    // every other non-empty layer must share this window (the model appends to all layers in
    // lockstep); a window lagging behind could be overwritten once this one wraps the ring
    for (size_t l = 0; l < kv->len.size(); ++l)
        if ((int)l != layer && kv->len[l] > 0 && (kv->len[l] != kv->len[layer] || kv->base[l] != kv->base[layer]))
            return fail(BEBELM_ERR_INVALID, "layer %zu's window differs from layer %d's; step plans need equal windows",
                        l, layer);
    DeviceGuard g(P->device);
    cudaStream_t s = 0;
    // give every ring entry a physical page
    if (kv->hi - kv->lo < kv->cap) {
        const long long add = kv->lo + kv->cap - kv->hi;
        if ((size_t)add > P->free_list.size())
            return fail(BEBELM_ERR_OOM, "page pool exhausted: a step plan needs %lld more pages, %zu free", add,
                        P->free_list.size());
        const long long old_hi = kv->hi;
        for (long long L = kv->hi; L < kv->lo + kv->cap; ++L) {
            kv->table[L % kv->cap] = P->free_list.back();
            P->free_list.pop_back();
        }
        kv->hi = kv->lo + kv->cap;
        TRY(upload_table(kv, old_hi, kv->hi, s));
    }
    auto* pl = new bebelm_step_plan();
    pl->kv = kv;
    pl->layer = layer;
    pl->n_heads = n_heads;
    long long b = kv->base[layer], n = kv->len[layer];
    if (n == 0 && b < kv->lo * kPageTokens) b = kv->lo * kPageTokens;
    pl->slot0 = b + n;
    pl->pos0 = (long long)kv->pos;
    pl->len0 = n;
    pl->window = (long long)window;
    // split plan for the largest window: the pages [base, base + window) can span
    const int group = n_heads / P->n_kv;
    pick_heads_per_cta(group, &pl->hpc, &pl->n_sub);
    const int NY = P->n_kv * pl->n_sub;
    const long long max_pages = (pl->window + kPageTokens - 1) / kPageTokens + 1;
    const long long target = (long long)P->num_sms * 2;  // two resident CTAs per SM, as run_decode
    long long per = std::max<long long>(1, (max_pages * NY + target - 1) / target);
    per = std::min<long long>(per, kDecodeMaxPagesPerSplit);
    pl->per = (int)per;
    pl->n_splits = (int)((max_pages + per - 1) / per);
    int rc = pl->state.ensure(sizeof(StepState), true, s);
    if (!rc) rc = pl->part.ensure(sizeof(float) * (size_t)pl->n_splits * NY * pl->hpc * (kHeadDim + 2), false, s);
    if (!rc) rc = pl->counters.ensure(sizeof(unsigned) * (size_t)NY, true, s);
    if (!rc && cudaStreamSynchronize(s) != cudaSuccess) rc = fail(BEBELM_ERR_CUDA, "step plan initialisation failed");
    if (rc) {
        pl->state.release();
        pl->part.release();
        pl->counters.release();
        delete pl;
        return rc;
    }
    kv->plans++;
    *out = pl;
    return 0;
}

}  // extern "C"

namespace {

// One step of a plan; with a peer group the outputs go to every rank's landing zone and a wait
// kernel gathers them into `out` ([world][n_heads*64]).
int plan_launch(bebelm_step_plan* pl, const bebelm_peer_group* grp, const float* q, const float* k, const float* v,
                const float* q_gain, const float* k_gain, float theta, float eps, float* out, void* stream) {
    if (!pl || !pl->kv) return fail(BEBELM_ERR_INVALID, "null step plan");
    if (!q || !k || !v || !q_gain || !k_gain || !out) return fail(BEBELM_ERR_INVALID, "null buffer");
    bebelm_kv* kv = pl->kv;
    bebelm_kv_pool* P = kv->pool;
    if (grp) {
        if (!grp->connected) return fail(BEBELM_ERR_INVALID, "peer group not connected");
        if (grp->device != P->device) return fail(BEBELM_ERR_INVALID, "cache and peer group are on different devices");
        if ((size_t)pl->n_heads * kHeadDim != grp->slice)
            return fail(BEBELM_ERR_INVALID, "n_heads*64 (%d) differs from the group's slice (%zu)", pl->n_heads * 64,
                        grp->slice);
    }
    DeviceGuard g(P->device);
    const int NY = P->n_kv * pl->n_sub;
    DecodeArgs a{};
    a.one.table = kv->d_table;
    a.one.cap = kv->cap;
    a.one.split0 = 0;
    a.one.n_splits = pl->n_splits;
    a.one.dep_slot = -1;
    a.n_seqs = 1;
    a.pv = P->view(pl->layer);
    a.q_raw = q;
    a.k_new = k;
    a.v_new = v;
    a.q_gain = q_gain;
    a.k_gain = k_gain;
    a.theta_scale = theta_scale_of(theta, kHeadDim);
    a.eps = eps;
    a.out = out;
    a.part_acc = pl->part.as<float>();
    a.part_ml = a.part_acc + (size_t)pl->n_splits * NY * pl->hpc * kHeadDim;
    a.counters = pl->counters.as<unsigned>();
    a.err = P->err.d;
    a.n_heads = pl->n_heads;
    a.n_kv = P->n_kv;
    a.group = pl->n_heads / P->n_kv;
    a.hpc = pl->hpc;
    a.n_sub = pl->n_sub;
    a.pages_per_split = pl->per;
    a.total_splits = pl->n_splits;
    a.scale_log2 = 0.125f * 1.4426950408889634f;
    a.pdl = 1;
    if (g_expire_waits > 0) {  // test hook (bebelm_debug_expire_next_wait)
        a.expire_wait = 1;
        --g_expire_waits;
    }
    a.step = pl->state.as<StepState>();
    a.step_slot0 = pl->slot0;
    a.step_pos0 = pl->pos0;
    a.step_len0 = pl->len0;
    a.step_window = pl->window;
    // Early reads need the previous decode launch to be another plan's, in the same stream
    // capture (or both uncaptured): a graph's first node must not rely on what preceded the
    // capture, since replays follow the graph's own last node.
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    unsigned long long cap_id = 0;
    CUDA_TRY(cudaStreamGetCaptureInfo(as_stream(stream), &cs, &cap_id));
    if (cs != cudaStreamCaptureStatusActive) cap_id = 0;
    a.step_prewait = P->last_plan != nullptr && P->last_plan != pl && P->last_capture == cap_id;
    if (grp) {
        // Between two gathered steps sits the previous step's wait kernel, an ordinary launch:
        // it starts once that decode grid has completed, and lets this grid start at once. So,
        // as between two plain plans, this plan's own previous step is complete when this grid
        // starts, and step_prewait (decided above) holds as it stands.
        a.peer_bufs = grp->d_bufs();
        a.peer_world = grp->world;
        a.peer_rank = grp->rank;
        a.peer_epoch = grp->d_epoch();
    }
    CUDA_TRY(launch_decode(a, as_stream(stream)));
    record_decode_out(as_stream(stream), a.out, grp ? SIZE_MAX : (size_t)pl->n_heads * kHeadDim * 4);
    P->last_plan = pl;
    P->last_capture = cap_id;
    if (grp) TRY(peer_gather_out(grp, P, out, as_stream(stream)));
    return 0;
}

}  // namespace

extern "C" {

int bebelm_step_plan_launch(bebelm_step_plan* pl, const float* q, const float* k, const float* v,
                            const float* q_gain, const float* k_gain, float theta, float eps, float* out,
                            void* stream) {
    return plan_launch(pl, nullptr, q, k, v, q_gain, k_gain, theta, eps, out, stream);
}

int bebelm_step_plan_launch_allgather(bebelm_step_plan* pl, bebelm_peer_group* g, const float* q, const float* k,
                                      const float* v, const float* q_gain, const float* k_gain, float theta,
                                      float eps, float* out, void* stream) {
    if (!g) return fail(BEBELM_ERR_INVALID, "null peer group");
    return plan_launch(pl, g, q, k, v, q_gain, k_gain, theta, eps, out, stream);
}

int bebelm_step_plan_steps(const bebelm_step_plan* pl, unsigned long long* n, void* stream) {
    if (!pl || !pl->kv || !n) return fail(BEBELM_ERR_INVALID, "null argument");
    DeviceGuard g(pl->kv->pool->device);
    cudaStream_t s = as_stream(stream);
    StepState st{};
    CUDA_TRY(cudaMemcpyAsync(&st, pl->state.p, sizeof(st), cudaMemcpyDeviceToHost, s));
    CUDA_TRY(cudaStreamSynchronize(s));
    *n = st.n;
    if (pl->kv->pool->err.read())
        return fail(BEBELM_ERR_TIMEOUT, "a device-side wait timed out; the plan's outputs are invalid");
    return 0;
}

int bebelm_step_plan_finish(bebelm_step_plan* pl, void* stream) {
    if (!pl || !pl->kv) return fail(BEBELM_ERR_INVALID, "null step plan");
    unsigned long long n = 0;
    const int rc = bebelm_step_plan_steps(pl, &n, stream);
    bebelm_kv* kv = pl->kv;
    if (rc == 0) {
        const long long end = pl->slot0 + (long long)n;  // one past the last appended slot
        const long long len = std::min(pl->len0 + (long long)n, pl->window);
        kv->base[pl->layer] = end - len;
        kv->len[pl->layer] = len;
        kv->pos = (size_t)(pl->pos0 + (long long)n);
        // the ring's pages now stand for the logical pages from the oldest live one on
        long long lo = LLONG_MAX;
        for (size_t l = 0; l < kv->len.size(); ++l)
            if (kv->len[l] > 0) lo = std::min(lo, kv->base[l] / kPageTokens);
        if (lo != LLONG_MAX && lo > kv->lo) {
            kv->lo = lo;
            kv->hi = lo + kv->cap;
        }
    }
    {
        DeviceGuard g(kv->pool->device);
        pl->state.release();
        pl->part.release();
        pl->counters.release();
        pl->lbuf.release();
    }
    kv->plans--;
    delete pl;
    return rc;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Quantized products of the weights feeding the path (the q/k/v/o projections).
// ---------------------------------------------------------------------------
namespace {

int check_ggml(int dtype, size_t n_in) {
    if (dtype != kGgmlF32 && dtype != kGgmlF16 && dtype != kGgmlQ4K && dtype != kGgmlQ6K)
        return fail(BEBELM_ERR_UNSUPPORTED, "weight dtype %d is not F32 (0), F16 (1), Q4_K (12) or Q6_K (14)", dtype);
    if ((dtype == kGgmlQ4K || dtype == kGgmlQ6K) && n_in % 256)
        return fail(BEBELM_ERR_INVALID, "n_in (%zu) must be a multiple of 256 for K-quant weights", n_in);
    return 0;
}

}  // namespace

extern "C" {

int bebelm_matmul(int dtype, const void* w, size_t n_in, size_t n_out, const float* x, size_t n_tokens, float* y,
                  int mem, void* stream) {
    TRY(check_mem(mem));
    TRY(check_ggml(dtype, n_in));
    if (n_out == 0 || n_tokens == 0) return 0;
    if (!y || (n_in && (!w || !x))) return fail(BEBELM_ERR_INVALID, "null buffer");
    int dev;
    TRY(current_device(&dev));
    cudaStream_t s = as_stream(stream);
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    bebelm_kv_pool* P = nullptr;
    TRY(scratch_pool(dev, &P));
    const size_t wbytes = ggml_row_bytes(dtype, n_in) * n_out, xn = n_in * n_tokens, yn = n_out * n_tokens;
    const void* dw = w;
    const float* dx = x;
    float* dy = y;
    if (mem == BEBELM_MEM_HOST) {
        void *a0, *a1, *o;
        Stage st[2] = {{w, wbytes, &a0}, {x, 4 * xn, &a1}};
        TRY(stage_in(P, st, 2, 4 * yn, &o, s));
        dw = a0;
        dx = static_cast<const float*>(a1);
        dy = static_cast<float*>(o);
    }
    int8_t* q8 = nullptr;
    float* q8s = nullptr;
    int* q8m = nullptr;
    if (dtype == kGgmlQ4K || dtype == kGgmlQ6K) {
        const size_t qb = (xn + 255) & ~size_t(255), sb = 4 * (xn / 256), mb = 4 * (xn / 32);
        TRY(P->q8.ensure(qb + ((sb + 255) & ~size_t(255)) + mb + 256, false, s));
        q8 = P->q8.as<int8_t>();
        q8s = reinterpret_cast<float*>(P->q8.as<char>() + qb);
        q8m = reinterpret_cast<int*>(P->q8.as<char>() + qb + ((sb + 255) & ~size_t(255)));
        CUDA_TRY(launch_quantize_q8(dx, n_in, n_tokens, q8, q8s, q8m, s));
    }
    CUDA_TRY(launch_qmatmul(dtype, static_cast<const uint8_t*>(dw), n_in, n_out, dx, n_tokens, q8, q8s, q8m, dy,
                             P->err.d, s));
    if (mem == BEBELM_MEM_HOST) return stage_out(P, dy, y, 4 * yn, s);
    return 0;
}

int bebelm_matvec(int dtype, const void* w, size_t n_in, size_t n_out, const float* x, float* y, int mem,
                  void* stream) {
    return bebelm_matmul(dtype, w, n_in, n_out, x, 1, y, mem, stream);
}

int bebelm_dequantize(int dtype, const void* data, size_t n_elements, float* out, int mem, void* stream) {
    TRY(check_mem(mem));
    TRY(check_ggml(dtype, n_elements));
    if (n_elements == 0) return 0;
    if (!data || !out) return fail(BEBELM_ERR_INVALID, "null buffer");
    int dev;
    TRY(current_device(&dev));
    cudaStream_t s = as_stream(stream);
    if (mem == BEBELM_MEM_DEVICE) {
        CUDA_TRY(launch_dequantize(dtype, static_cast<const uint8_t*>(data), n_elements, out, s));
        return 0;
    }
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    bebelm_kv_pool* P = nullptr;
    TRY(scratch_pool(dev, &P));
    void *a0, *o;
    Stage st[1] = {{data, ggml_row_bytes(dtype, n_elements), &a0}};
    TRY(stage_in(P, st, 1, 4 * n_elements, &o, s));
    CUDA_TRY(launch_dequantize(dtype, static_cast<const uint8_t*>(a0), n_elements, static_cast<float*>(o), s));
    return stage_out(P, o, out, 4 * n_elements, s);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// The whole attention operator of a layer: projections + the fused step / prefill + output
// projection, on device-resident GGML weights (src/model.rs:430-455 attn_step, 224-258
// attn_batch).
// ---------------------------------------------------------------------------
struct bebelm_attn_weights {
    int device = 0, n_heads = 0, n_kv = 0;
    size_t hidden = 0;
    int dt[4] = {0, 0, 0, 0};  // q, k, v, o
    DevBuf w[4], gains;        // gains: q_gain[64] then k_gain[64]
};

namespace {

// Q8 activations of x [t][n_in] in the pool's scratch (for K-quant weights)
struct Q8View {
    int8_t* q = nullptr;
    float* sc = nullptr;
    int* sm = nullptr;
};

int quantize_into_scratch(bebelm_kv_pool* P, const float* x, size_t n_in, size_t t, Q8View* v, cudaStream_t s) {
    const size_t xn = n_in * t, qb = (xn + 255) & ~size_t(255), sb = (4 * (xn / 256) + 255) & ~size_t(255);
    TRY(P->q8.ensure(qb + sb + 4 * (xn / 32) + 256, false, s));
    v->q = P->q8.as<int8_t>();
    v->sc = reinterpret_cast<float*>(P->q8.as<char>() + qb);
    v->sm = reinterpret_cast<int*>(P->q8.as<char>() + qb + sb);
    CUDA_TRY(launch_quantize_q8(x, n_in, t, v->q, v->sc, v->sm, s));
    return 0;
}

bool is_kquant(int dt) { return dt == kGgmlQ4K || dt == kGgmlQ6K; }

// y = W x for the weights of one projection; x already quantized in q8 when needed
int project(const bebelm_attn_weights* W, int which, size_t n_in, size_t n_out, const float* x, size_t t,
            const Q8View& q8, float* y, int* err, cudaStream_t s) {
    CUDA_TRY(launch_qmatmul(W->dt[which], W->w[which].as<uint8_t>(), n_in, n_out, x, t, q8.q, q8.sc, q8.sm, y, err, s));
    return 0;
}

int check_weights(const bebelm_kv* kv, const bebelm_attn_weights* W) {
    if (!W) return fail(BEBELM_ERR_INVALID, "null weights");
    if (W->device != kv->pool->device) return fail(BEBELM_ERR_INVALID, "weights and cache are on different devices");
    if (W->n_kv != kv->pool->n_kv)
        return fail(BEBELM_ERR_INVALID, "weights have %d kv heads, the cache %d", W->n_kv, kv->pool->n_kv);
    return 0;
}

// x [t][hidden] (device) -> q [t][nq], k/v [t][nkv] into the pool's projection scratch
int project_qkv(bebelm_kv_pool* P, const bebelm_attn_weights* W, const float* dx, size_t t, float** q, float** k,
                float** v, float** attn, cudaStream_t s) {
    const size_t nq = (size_t)W->n_heads * kHeadDim, nkv = (size_t)W->n_kv * kHeadDim;
    TRY(P->proj.ensure(4 * t * (2 * nq + 2 * nkv) + 1024, false, s));
    *q = P->proj.as<float>();
    *k = *q + t * nq;
    *v = *k + t * nkv;
    *attn = *v + t * nkv;
    Q8View q8;
    if (is_kquant(W->dt[0]) || is_kquant(W->dt[1]) || is_kquant(W->dt[2]))
        TRY(quantize_into_scratch(P, dx, W->hidden, t, &q8, s));
    // the k and v projections (n_kv*64 rows: too few CTAs to fill the GPU) run on the pool's
    // side stream beside the q projection, forked after the quantization and joined before
    // anything reads them
    if (!P->side) {
        CUDA_TRY(cudaStreamCreateWithFlags(&P->side, cudaStreamNonBlocking));
        CUDA_TRY(cudaEventCreateWithFlags(&P->ev_fork, cudaEventDisableTiming));
        CUDA_TRY(cudaEventCreateWithFlags(&P->ev_join, cudaEventDisableTiming));
    }
    CUDA_TRY(cudaEventRecord(P->ev_fork, s));
    CUDA_TRY(cudaStreamWaitEvent(P->side, P->ev_fork, 0));
    TRY(project(W, 1, W->hidden, nkv, dx, t, q8, *k, P->err.d, P->side));
    TRY(project(W, 2, W->hidden, nkv, dx, t, q8, *v, P->err.d, P->side));
    CUDA_TRY(cudaEventRecord(P->ev_join, P->side));
    TRY(project(W, 0, W->hidden, nq, dx, t, q8, *q, P->err.d, s));
    CUDA_TRY(cudaStreamWaitEvent(s, P->ev_join, 0));
    return 0;
}

// One token: q/k/v = W x in one launch (x quantized inside it), and out = W_o attn in one.
int project_token(const bebelm_attn_weights* W, const float* x, float* q, float* k, float* v, cudaStream_t s) {
    const size_t nq = (size_t)W->n_heads * kHeadDim, nkv = (size_t)W->n_kv * kHeadDim;
    QmvSegs sg{};
    sg.n = 3;
    float* ys[3] = {q, k, v};
    const size_t no[3] = {nq, nkv, nkv};
    for (int i = 0; i < 3; ++i) {
        sg.dtype[i] = W->dt[i];
        sg.w[i] = W->w[i].as<uint8_t>();
        sg.row_bytes[i] = ggml_row_bytes(W->dt[i], W->hidden);
        sg.n_out[i] = no[i];
        sg.y[i] = ys[i];
    }
    CUDA_TRY(launch_qmv_multi(sg, x, W->hidden, s));
    return 0;
}

int project_token_out(const bebelm_attn_weights* W, const float* attn, float* out, cudaStream_t s) {
    const size_t nq = (size_t)W->n_heads * kHeadDim;
    QmvSegs sg{};
    sg.n = 1;
    sg.dtype[0] = W->dt[3];
    sg.w[0] = W->w[3].as<uint8_t>();
    sg.row_bytes[0] = ggml_row_bytes(W->dt[3], nq);
    sg.n_out[0] = W->hidden;
    sg.y[0] = out;
    CUDA_TRY(launch_qmv_multi(sg, attn, nq, s));
    return 0;
}

int project_out(bebelm_kv_pool* P, const bebelm_attn_weights* W, const float* attn, size_t t, float* dout,
                cudaStream_t s) {
    const size_t nq = (size_t)W->n_heads * kHeadDim;
    Q8View q8;
    if (is_kquant(W->dt[3])) TRY(quantize_into_scratch(P, attn, nq, t, &q8, s));
    return project(W, 3, nq, W->hidden, attn, t, q8, dout, P->err.d, s);
}

}  // namespace

extern "C" {

int bebelm_attn_weights_create(int device, int n_heads, int n_kv_heads, size_t hidden, int dtype_q, const void* wq,
                               int dtype_k, const void* wk, int dtype_v, const void* wv, int dtype_o, const void* wo,
                               const float* q_gain, const float* k_gain, bebelm_attn_weights** out) {
    if (!out) return fail(BEBELM_ERR_INVALID, "out is null");
    *out = nullptr;
    TRY(check_geometry(n_heads, n_kv_heads));
    if (!wq || !wk || !wv || !wo || !q_gain || !k_gain) return fail(BEBELM_ERR_INVALID, "null buffer");
    const size_t nq = (size_t)n_heads * kHeadDim, nkv = (size_t)n_kv_heads * kHeadDim;
    const int dts[4] = {dtype_q, dtype_k, dtype_v, dtype_o};
    const size_t n_in[4] = {hidden, hidden, hidden, nq}, n_out[4] = {nq, nkv, nkv, hidden};
    for (int i = 0; i < 4; ++i) TRY(check_ggml(dts[i], n_in[i]));
    if (hidden > 8192 || nq > 8192)
        return fail(BEBELM_ERR_UNSUPPORTED, "hidden (%zu) and n_heads*64 (%zu) must be at most 8192", hidden, nq);
    int n_dev = 0;
    CUDA_TRY(cudaGetDeviceCount(&n_dev));
    if (device < 0 || device >= n_dev) return fail(BEBELM_ERR_INVALID, "device %d not present", device);
    DeviceGuard g(device);
    auto* W = new bebelm_attn_weights();
    W->device = device;
    W->n_heads = n_heads;
    W->n_kv = n_kv_heads;
    W->hidden = hidden;
    const void* src[4] = {wq, wk, wv, wo};
    int rc = 0;
    for (int i = 0; i < 4 && !rc; ++i) {
        W->dt[i] = dts[i];
        const size_t bytes = ggml_row_bytes(dts[i], n_in[i]) * n_out[i];
        rc = W->w[i].ensure(bytes);
        if (!rc && cudaMemcpy(W->w[i].p, src[i], bytes, cudaMemcpyHostToDevice) != cudaSuccess)
            rc = fail(BEBELM_ERR_CUDA, "uploading weight %d failed", i);
    }
    if (!rc) rc = W->gains.ensure(2 * 64 * sizeof(float));
    if (!rc && (cudaMemcpy(W->gains.p, q_gain, 64 * sizeof(float), cudaMemcpyHostToDevice) != cudaSuccess ||
                cudaMemcpy(W->gains.as<float>() + 64, k_gain, 64 * sizeof(float), cudaMemcpyHostToDevice) != cudaSuccess))
        rc = fail(BEBELM_ERR_CUDA, "uploading the norm gains failed");
    if (rc) {
        for (auto& b : W->w) b.release();
        W->gains.release();
        delete W;
        return rc;
    }
    *out = W;
    return 0;
}

int bebelm_attn_weights_destroy(bebelm_attn_weights* W) {
    if (!W) return 0;
    DeviceGuard g(W->device);
    cudaDeviceSynchronize();
    for (auto& b : W->w) b.release();
    W->gains.release();
    delete W;
    return 0;
}

int bebelm_attn_layer_step(bebelm_kv* kv, int layer, const bebelm_attn_weights* W, const float* x, size_t pos,
                           float theta, float eps, float* out, int mem, void* stream) {
    TRY(validate_layer(kv, layer));
    TRY(check_mem(mem));
    TRY(check_weights(kv, W));
    if (!x || !out) return fail(BEBELM_ERR_INVALID, "null buffer");
    bebelm_kv_pool* P = kv->pool;
    DeviceGuard g(P->device);
    cudaStream_t s = as_stream(stream);
    const float* dx = x;
    float* dout = out;
    if (mem == BEBELM_MEM_HOST) {
        void *a0, *o;
        Stage st[1] = {{x, 4 * W->hidden, &a0}};
        TRY(stage_in(P, st, 1, 4 * W->hidden, &o, s));
        dx = static_cast<const float*>(a0);
        dout = static_cast<float*>(o);
    }
    const size_t nq = (size_t)W->n_heads * kHeadDim, nkv = (size_t)W->n_kv * kHeadDim;
    TRY(P->proj.ensure(4 * (2 * nq + 2 * nkv) + 1024, false, s));
    float* q = P->proj.as<float>();
    float *k = q + nq, *v = k + nkv, *attn = v + nkv;
    TRY(project_token(W, dx, q, k, v, s));
    long long slot0 = 0;
    TRY(reserve(kv, layer, 1, &slot0, s));
    const FusedStep fs{q, k, v, W->gains.as<float>(), W->gains.as<float>() + 64, theta_scale_of(theta, kHeadDim), eps};
    std::vector<Window> w{{kv, kv->base[layer], kv->len[layer], slot0, (long long)pos}};
    TRY(run_decode(P, w, layer, W->n_heads, nullptr, attn, 0.125f, &fs, s));
    TRY(project_token_out(W, attn, dout, s));
    if (mem == BEBELM_MEM_HOST) return stage_out(P, dout, out, 4 * W->hidden, s);
    return 0;
}

int bebelm_attn_layer_batch(bebelm_kv* kv, int layer, const bebelm_attn_weights* W, const float* x, size_t t,
                            size_t pos0, int tensor_cores, float theta, float eps, float* out, int mem, void* stream) {
    TRY(validate_layer(kv, layer));
    TRY(check_mem(mem));
    TRY(check_weights(kv, W));
    if (t == 0) return 0;
    if (!x || !out) return fail(BEBELM_ERR_INVALID, "null buffer");
    bebelm_kv_pool* P = kv->pool;
    DeviceGuard g(P->device);
    cudaStream_t s = as_stream(stream);
    const size_t xn = t * W->hidden;
    const float* dx = x;
    float* dout = out;
    if (mem == BEBELM_MEM_HOST) {
        void *a0, *o;
        Stage st[1] = {{x, 4 * xn, &a0}};
        TRY(stage_in(P, st, 1, 4 * xn, &o, s));
        dx = static_cast<const float*>(a0);
        dout = static_cast<float*>(o);
    }
    float *q, *k, *v, *attn;
    TRY(project_qkv(P, W, dx, t, &q, &k, &v, &attn, s));
    TRY(prefill_device(kv, layer, W->n_heads, q, k, v, false, tensor_cores != 0, t, pos0, W->gains.as<float>(),
                       W->gains.as<float>() + 64, theta, eps, attn, s));
    TRY(project_out(P, W, attn, t, dout, s));
    if (mem == BEBELM_MEM_HOST) return stage_out(P, dout, out, 4 * xn, s);
    return 0;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Whole-operator step plans: a plan's decode wrapped in the layer's projections, all on
// scratch the plan owns, so a token's attention layers can be captured in one graph.
// ---------------------------------------------------------------------------
namespace {

struct LayerScratch {
    float *q, *k, *v, *attn;
    int8_t* q8;
    float* q8s;
    int* q8m;
};

LayerScratch layer_scratch(const bebelm_step_plan* pl) {
    const bebelm_attn_weights* W = pl->W;
    const size_t nq = (size_t)W->n_heads * kHeadDim, nkv = (size_t)W->n_kv * kHeadDim;
    const size_t nx = std::max(W->hidden, nq);
    LayerScratch L;
    L.q = pl->lbuf.as<float>();
    L.k = L.q + nq;
    L.v = L.k + nkv;
    L.attn = L.v + nkv;
    char* b = reinterpret_cast<char*>(L.attn + nq);
    L.q8 = reinterpret_cast<int8_t*>(b);
    L.q8s = reinterpret_cast<float*>(b + ((nx + 255) & ~size_t(255)));
    L.q8m = reinterpret_cast<int*>(b + ((nx + 255) & ~size_t(255)) + ((4 * (nx / 256) + 255) & ~size_t(255)));
    return L;
}

size_t layer_scratch_bytes(const bebelm_attn_weights* W) {
    const size_t nq = (size_t)W->n_heads * kHeadDim, nkv = (size_t)W->n_kv * kHeadDim;
    const size_t nx = std::max(W->hidden, nq);
    return 4 * (2 * nq + 2 * nkv) + ((nx + 255) & ~size_t(255)) + ((4 * (nx / 256) + 255) & ~size_t(255)) +
           4 * (nx / 32) + 256;
}

}  // namespace

extern "C" {

int bebelm_step_plan_create_layer(bebelm_kv* kv, int layer, const bebelm_attn_weights* w, size_t window,
                                  bebelm_step_plan** out) {
    if (!out) return fail(BEBELM_ERR_INVALID, "out is null");
    *out = nullptr;
    if (!kv || !kv->pool) return fail(BEBELM_ERR_INVALID, "null cache handle");
    TRY(check_weights(kv, w));
    TRY(bebelm_step_plan_create(kv, layer, w->n_heads, window, out));
    bebelm_step_plan* pl = *out;
    pl->W = w;
    int rc;
    {
        DeviceGuard g(kv->pool->device);
        rc = pl->lbuf.ensure(layer_scratch_bytes(w), true);
        if (!rc && cudaDeviceSynchronize() != cudaSuccess) rc = fail(BEBELM_ERR_CUDA, "step plan scratch failed");
    }
    if (rc) {
        bebelm_step_plan_finish(pl, nullptr);
        *out = nullptr;
        return rc;
    }
    return 0;
}

int bebelm_step_plan_launch_layer(bebelm_step_plan* pl, const float* x, float theta, float eps, float* out,
                                  void* stream) {
    if (!pl || !pl->kv) return fail(BEBELM_ERR_INVALID, "null step plan");
    if (!pl->W) return fail(BEBELM_ERR_INVALID, "the plan was not created with layer weights");
    if (!x || !out) return fail(BEBELM_ERR_INVALID, "null buffer");
    const bebelm_attn_weights* W = pl->W;
    DeviceGuard g(pl->kv->pool->device);
    cudaStream_t s = as_stream(stream);
    const LayerScratch L = layer_scratch(pl);
    TRY(project_token(W, x, L.q, L.k, L.v, s));
    TRY(bebelm_step_plan_launch(pl, L.q, L.k, L.v, W->gains.as<float>(), W->gains.as<float>() + 64, theta, eps,
                                L.attn, stream));
    return project_token_out(W, L.attn, out, s);
}

// ---------------------------------------------------------------- logits head ---

constexpr size_t kHeadCandSlots = 1024;  // >= SMs per device
constexpr size_t kHeadCandBytes = 2 * 4 * kHeadCandSlots + 256;

struct bebelm_head {
    int device = 0, dtype = 0;
    size_t hidden = 0, vocab = 0;
    DevBuf w, gain, normed, logits, token, cand;  // cand: per-SM argmax candidates + counter
    ErrWord err;  // a bounded wait of the streaming matvec that gave up
};

int bebelm_head_create(int device, int dtype, const void* token_embd, size_t hidden, size_t vocab,
                       const float* norm_gain, bebelm_head** out) {
    if (!out) return fail(BEBELM_ERR_INVALID, "out is null");
    *out = nullptr;
    if (!token_embd || !norm_gain) return fail(BEBELM_ERR_INVALID, "null buffer");
    TRY(check_ggml(dtype, hidden));
    if (hidden == 0 || hidden > 8192) return fail(BEBELM_ERR_UNSUPPORTED, "hidden (%zu) must be 1..8192", hidden);
    if (vocab == 0 || vocab >= (1ull << 32)) return fail(BEBELM_ERR_INVALID, "vocab (%zu) must be 1..2^32-1", vocab);
    int n_dev = 0;
    CUDA_TRY(cudaGetDeviceCount(&n_dev));
    if (device < 0 || device >= n_dev) return fail(BEBELM_ERR_INVALID, "device %d not present", device);
    DeviceGuard g(device);
    auto* H = new bebelm_head();
    H->device = device;
    H->dtype = dtype;
    H->hidden = hidden;
    H->vocab = vocab;
    const size_t wbytes = ggml_row_bytes(dtype, hidden) * vocab;
    int rc = H->w.ensure(wbytes);
    if (!rc && cudaMemcpy(H->w.p, token_embd, wbytes, cudaMemcpyHostToDevice) != cudaSuccess)
        rc = fail(BEBELM_ERR_CUDA, "uploading token_embd failed");
    if (!rc) rc = H->gain.ensure(hidden * sizeof(float));
    if (!rc && cudaMemcpy(H->gain.p, norm_gain, hidden * sizeof(float), cudaMemcpyHostToDevice) != cudaSuccess)
        rc = fail(BEBELM_ERR_CUDA, "uploading the norm gain failed");
    if (!rc) rc = H->normed.ensure(hidden * sizeof(float));
    if (!rc) rc = H->logits.ensure(vocab * sizeof(float));
    if (!rc) rc = H->token.ensure(256);
    if (!rc) rc = H->err.ensure();
    if (!rc) rc = H->cand.ensure(kHeadCandBytes, true);
    if (rc) {
        H->w.release();
        H->gain.release();
        H->normed.release();
        H->logits.release();
        H->token.release();
        H->err.release();
        H->cand.release();
        delete H;
        return rc;
    }
    *out = H;
    return 0;
}

int bebelm_head_destroy(bebelm_head* H) {
    if (!H) return 0;
    DeviceGuard g(H->device);
    cudaDeviceSynchronize();
    H->w.release();
    H->gain.release();
    H->normed.release();
    H->logits.release();
    H->token.release();
    H->err.release();
    H->cand.release();
    delete H;
    return 0;
}

int bebelm_head_logits(bebelm_head* H, const float* h, float eps, float* logits, uint32_t* token, int mem,
                       void* stream) {
    if (!H) return fail(BEBELM_ERR_INVALID, "null head");
    TRY(check_mem(mem));
    if (!h) return fail(BEBELM_ERR_INVALID, "null buffer");
    DeviceGuard g(H->device);
    cudaStream_t s = as_stream(stream);
    // a device-side timeout of an earlier device-memory call is reported here
    if (H->err.read()) {
        const int e = H->err.read();
        H->err.clear();
        return fail(BEBELM_ERR_TIMEOUT, "a device-side wait of the logits head timed out (code %d)", e);
    }
    auto run = [&](const float* dh, float* dlogits, uint32_t* dtoken) -> int {
        // vocab-sized K-quant matrices: one streaming launch (norm, matvec, argmax); otherwise
        // the norm, the lane matvec and the argmax as three launches (same bits)
        if (H->vocab >= 8192) {
            float* cv = H->cand.as<float>();
            const cudaError_t se = launch_head_stream(
                H->dtype, H->w.as<uint8_t>(), H->vocab, dh, H->gain.as<float>(), eps, H->hidden, dlogits, dtoken, cv,
                reinterpret_cast<uint32_t*>(cv + kHeadCandSlots), reinterpret_cast<unsigned*>(cv + 2 * kHeadCandSlots),
                H->err.d, s);
            if (se != cudaErrorNotSupported) {
                CUDA_TRY(se);
                return 0;
            }
        }
        CUDA_TRY(launch_rmsnorm_row(dh, H->gain.as<float>(), (int)H->hidden, eps, H->normed.as<float>(), s));
        QmvSegs sg{};
        sg.n = 1;
        sg.dtype[0] = H->dtype;
        sg.w[0] = H->w.as<uint8_t>();
        sg.row_bytes[0] = ggml_row_bytes(H->dtype, H->hidden);
        sg.n_out[0] = H->vocab;
        sg.y[0] = dlogits;
        CUDA_TRY(launch_qmv_multi(sg, H->normed.as<float>(), H->hidden, s));
        if (dtoken) CUDA_TRY(launch_greedy(dlogits, H->vocab, nullptr, 0, 1.0f, nullptr, dtoken, s));
        return 0;
    };
    if (mem == BEBELM_MEM_DEVICE)
        return run(h, logits ? logits : H->logits.as<float>(), token);
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    bebelm_kv_pool* P = nullptr;
    TRY(scratch_pool(H->device, &P));
    const size_t lbytes = logits ? 4 * H->vocab : 0, out_bytes = 256 + lbytes;
    void *a0, *o;
    Stage st[1] = {{h, 4 * H->hidden, &a0}};
    TRY(stage_in(P, st, 1, out_bytes, &o, s));
    char* dout = static_cast<char*>(o);
    TRY(run(static_cast<const float*>(a0), logits ? reinterpret_cast<float*>(dout + 256) : H->logits.as<float>(),
            reinterpret_cast<uint32_t*>(dout)));
    std::vector<char> back(out_bytes);
    TRY(stage_out(P, o, back.data(), out_bytes, s));
    if (H->err.read()) {
        const int e = H->err.read();
        H->err.clear();
        return fail(BEBELM_ERR_TIMEOUT, "a device-side wait of the logits head timed out (code %d)", e);
    }
    if (token) std::memcpy(token, back.data(), 4);
    if (logits) std::memcpy(logits, back.data() + 256, lbytes);
    return 0;
}

int bebelm_sample_greedy(float* logits, size_t n, const uint32_t* history, size_t n_history, float repeat_penalty,
                         uint32_t* token, int mem, void* stream) {
    TRY(check_mem(mem));
    if (!logits || !token || (n_history && !history)) return fail(BEBELM_ERR_INVALID, "null buffer");
    if (n == 0 || n >= (1ull << 32)) return fail(BEBELM_ERR_INVALID, "n (%zu) must be 1..2^32-1", n);
    const bool pen = repeat_penalty != 1.0f && n_history > 0;
    if (pen && mem == BEBELM_MEM_HOST)
        for (size_t i = 0; i < n_history; ++i)
            if (history[i] >= n) return fail(BEBELM_ERR_INVALID, "history token %u out of range", history[i]);
    int dev;
    TRY(current_device(&dev));
    cudaStream_t s = as_stream(stream);
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    bebelm_kv_pool* P = nullptr;
    TRY(scratch_pool(dev, &P));
    if (pen) TRY(P->sample.ensure((n + 31) / 32 * 4, false, s));
    uint32_t* bitmap = pen ? P->sample.as<uint32_t>() : nullptr;
    if (mem == BEBELM_MEM_DEVICE) {
        CUDA_TRY(launch_greedy(logits, n, history, pen ? n_history : 0, repeat_penalty, bitmap, token, s));
        return 0;
    }
    void *a0, *a1, *o;
    Stage st[2] = {{logits, 4 * n, &a0}, {pen ? history : nullptr, pen ? 4 * n_history : 0, &a1}};
    TRY(stage_in(P, st, 2, 4, &o, s));
    CUDA_TRY(launch_greedy(static_cast<float*>(a0), n, static_cast<const uint32_t*>(a1), pen ? n_history : 0,
                           repeat_penalty, bitmap, static_cast<uint32_t*>(o), s));
    TRY(stage_out(P, o, token, 4, s));
    // the penalty rewrites the seen tokens' logits in place, as the reference's sampler does
    if (pen) CUDA_TRY(cudaMemcpy(logits, a0, 4 * n, cudaMemcpyDeviceToHost));
    return 0;
}

}  // extern "C"
