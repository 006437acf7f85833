/*
 * CPU ORACLE — test infrastructure only, never part of the product path.
 *
 * A plain-C restatement of BebeLM's attention arithmetic (reference crate
 * maximecb/bebelm 0.3.6, Rust). Only the test suite, the smoke check and the
 * CPU-baseline leg of bench.py load this library; the CUDA library never does.
 *
 * Each function cites the reference file:line it restates. Build flags are
 * -O2 -ffp-contract=off so that every a*b+c stays two roundings unless the
 * reference itself fuses (the `dot` below calls fmaf where `wide::f32x8::mul_add`
 * fuses on an FMA-capable x86 host).
 *
 * Pinning: the elementary kernels are checked against every known-answer test
 * the reference's own unit tests hold (attention.rs:61-92, softmax.rs:35-114,
 * rmsnorm.rs:27-117, rope.rs:37-77, cache.rs:61-77, matmul.rs:1064-1086), see
 * tests/golden/reference_kats.json. The reference cannot be compiled here (no
 * Rust toolchain), so the horizontal-add order of `wide 0.7.33`'s
 * `f32x8::reduce_add` is not pinned bit-for-bit: the restatement below picks a
 * pairwise order and parity against the GPU is asserted to tolerance.
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <pthread.h>
#include <unistd.h>

/* ---------------------------------------------------------------- PRNG --- */
/* Seeded inputs shared by tests and the CPU baseline: SplitMix64 -> uniform
 * double in (0,1) -> Box-Muller -> N(0,1) float. Deterministic everywhere. */
static uint64_t splitmix64(uint64_t* s) {
    uint64_t z = (*s += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

static double uniform01(uint64_t* s) {
    /* 53 random bits, shifted off zero */
    return ((double)(splitmix64(s) >> 11) + 0.5) * (1.0 / 9007199254740992.0);
}

void orc_fill_normal(uint64_t seed, size_t n, float mean, float stddev, float* out) {
    uint64_t s = seed;
    size_t i = 0;
    while (i < n) {
        double u1 = uniform01(&s), u2 = uniform01(&s);
        double r = sqrt(-2.0 * log(u1));
        double a = 6.283185307179586 * u2;
        out[i++] = (float)(mean + stddev * r * cos(a));
        if (i < n) out[i++] = (float)(mean + stddev * r * sin(a));
    }
}

void orc_fill_uniform_int(uint64_t seed, size_t n, int64_t lo, int64_t hi, int64_t* out) {
    uint64_t s = seed;
    uint64_t span = (uint64_t)(hi - lo + 1);
    for (size_t i = 0; i < n; ++i) out[i] = lo + (int64_t)(splitmix64(&s) % span);
}

/* ----------------------------------------------------------------- dot --- */
/* src/kernels/matmul.rs:36-65. Four f32x8 accumulators fed by mul_add (fused on
 * an FMA host, .cargo/config.toml:11-12 builds with target-cpu=native), an
 * 8-wide cleanup loop, then ((acc0+acc1)+(acc2+acc3)).reduce_add() and a scalar
 * tail `sum += a*b` (unfused). reduce_add order (unpinned, see header): lanes
 * i and i+4 added, then (0,2),(1,3), then the two halves. */
static float reduce_add8(const float v[8]) {
    float h0 = v[0] + v[4], h1 = v[1] + v[5], h2 = v[2] + v[6], h3 = v[3] + v[7];
    float q0 = h0 + h2, q1 = h1 + h3;
    return q0 + q1;
}

float orc_dot(const float* a, const float* b, size_t n) {
    float acc[4][8];
    memset(acc, 0, sizeof acc);
    size_t i = 0;
    while (i + 32 <= n) {
        for (int r = 0; r < 4; ++r)
            for (int l = 0; l < 8; ++l)
                acc[r][l] = fmaf(a[i + 8 * r + l], b[i + 8 * r + l], acc[r][l]);
        i += 32;
    }
    while (i + 8 <= n) {
        for (int l = 0; l < 8; ++l) acc[0][l] = fmaf(a[i + l], b[i + l], acc[0][l]);
        i += 8;
    }
    float s01[8], s23[8], s[8];
    for (int l = 0; l < 8; ++l) {
        s01[l] = acc[0][l] + acc[1][l];
        s23[l] = acc[2][l] + acc[3][l];
        s[l] = s01[l] + s23[l];
    }
    float sum = reduce_add8(s);
    while (i < n) {
        float p = a[i] * b[i];
        sum += p;
        ++i;
    }
    return sum;
}

/* ------------------------------------------------------------- softmax --- */
/* src/kernels/softmax.rs:9-22: max (first of ties kept by `a >= b`), f32 exp of
 * (x - max), Σ in f64 of the widened f32 exps, inv = (1/sum) narrowed to f32,
 * x *= inv. Empty input is a no-op. */
void orc_softmax(float* x, size_t n) {
    if (n == 0) return;
    float mx = x[0];
    for (size_t i = 1; i < n; ++i) mx = (mx >= x[i]) ? mx : x[i];
    double sum = 0.0;
    for (size_t i = 0; i < n; ++i) {
        x[i] = expf(x[i] - mx);
        sum += (double)x[i];
    }
    float inv = (float)(1.0 / sum);
    for (size_t i = 0; i < n; ++i) x[i] *= inv;
}

/* ------------------------------------------------------------- rmsnorm --- */
/* src/kernels/rmsnorm.rs:10-21: ss = Σ (float)(x*x) widened to f64, mean =
 * (float)(ss/n), scale = 1/sqrtf(mean+eps), out = (x*scale)*g. */
void orc_rmsnorm(const float* x, const float* gain, float eps, float* out, size_t n) {
    double ss = 0.0;
    for (size_t i = 0; i < n; ++i) {
        float sq = x[i] * x[i];
        ss += (double)sq;
    }
    float mean = (float)(ss / (double)n);
    float scale = 1.0f / sqrtf(mean + eps);
    for (size_t i = 0; i < n; ++i) {
        float t = x[i] * scale;
        out[i] = t * gain[i];
    }
}

/* ----------------------------------------------------------------- rope --- */
/* src/kernels/rope.rs:16-29: NEOX split-half pairs (i, i+d/2); theta_scale =
 * powf(base, -2/d); theta starts at (float)pos and is multiplied by theta_scale
 * after each pair (iterative, as ggml does). Rust's f32::sin_cos is sinf/cosf. */
void orc_rope_neox(float* x, size_t d, size_t pos, float freq_base) {
    size_t half = d / 2;
    float theta_scale = powf(freq_base, -2.0f / (float)d);
    float theta = (float)pos;
    for (size_t i = 0; i < half; ++i) {
        float s = sinf(theta), c = cosf(theta);
        float a = x[i], b = x[i + half];
        float as = a * s, ac = a * c, bs = b * s, bc = b * c;
        x[i] = ac - bs;
        x[i + half] = as + bc;
        theta *= theta_scale;
    }
}

/* ------------------------------------------------------ norm_rope_heads --- */
/* src/model.rs:600-608: per head, rmsnorm into a temporary, copy back, then RoPE
 * at `pos`. The reference fixes eps = RMS_EPS (1e-5) and base = ROPE_THETA
 * (5e6, src/config.rs:31-32); both are parameters here. */
void orc_norm_rope_heads(float* buf, int n_heads, int head_dim, const float* gain,
                         size_t pos, float theta, float eps) {
    float tmp[4096];
    for (int h = 0; h < n_heads; ++h) {
        float* head = buf + (size_t)h * head_dim;
        orc_rmsnorm(head, gain, eps, tmp, (size_t)head_dim);
        memcpy(head, tmp, sizeof(float) * (size_t)head_dim);
        orc_rope_neox(head, (size_t)head_dim, pos, theta);
    }
}

/* ----------------------------------------------------- attention_decode --- */
/* One query head against n_ctx keys: src/kernels/attention.rs:37-54 for a
 * single h (scores via dot * scale, softmax, then out += w*v in j order with a
 * separate multiply and add). `scores` is caller scratch of n_ctx floats. */
static void attend_head(const float* qv, const float* k, const float* v, size_t n_ctx,
                        int n_kv_heads, int head_dim, int kv, float scale,
                        float* scores, float* outv) {
    for (size_t j = 0; j < n_ctx; ++j) {
        const float* kj = k + (j * (size_t)n_kv_heads + (size_t)kv) * (size_t)head_dim;
        scores[j] = orc_dot(qv, kj, (size_t)head_dim) * scale;
    }
    orc_softmax(scores, n_ctx);
    for (int d = 0; d < head_dim; ++d) outv[d] = 0.0f;
    for (size_t j = 0; j < n_ctx; ++j) {
        const float* vj = v + (j * (size_t)n_kv_heads + (size_t)kv) * (size_t)head_dim;
        float w = scores[j];
        for (int d = 0; d < head_dim; ++d) {
            float p = w * vj[d];
            outv[d] += p;
        }
    }
}

/* src/kernels/attention.rs:17-55. q/out [n_heads*head_dim]; k/v token-major
 * [n_ctx][n_kv_heads][head_dim]; kv head = h / (n_heads/n_kv_heads); scale =
 * 1/sqrtf(head_dim). Returns 0, or -1 on bad geometry (the reference panics in
 * debug builds). n_ctx == 0 leaves zeros (softmax of nothing, nothing added). */
int orc_attention_decode(const float* q, const float* k, const float* v, size_t n_ctx,
                         int n_heads, int n_kv_heads, int head_dim, float* out) {
    if (n_heads <= 0 || n_kv_heads <= 0 || head_dim <= 0 || n_heads % n_kv_heads) return -1;
    float scale = 1.0f / sqrtf((float)head_dim);
    int group = n_heads / n_kv_heads;
    float* scores = (float*)malloc(sizeof(float) * (n_ctx ? n_ctx : 1));
    if (!scores) return -2;
    for (int h = 0; h < n_heads; ++h)
        attend_head(q + (size_t)h * head_dim, k, v, n_ctx, n_kv_heads, head_dim, h / group,
                    scale, scores, out + (size_t)h * head_dim);
    free(scores);
    return 0;
}

/* Harness extension (NOT reference behaviour): a tiny pthread parallel-for
 * used by the multi-core CPU baseline. Work items are independent (token, head)
 * attention problems, so spreading them leaves each item's arithmetic — and
 * hence the result — bit-identical to the serial functions. */
typedef struct {
    const float *q, *k, *v;
    float* out;
    size_t n_ctx_base; /* keys seen by every item, plus i+1 when causal */
    int causal;        /* 1: item i attends n_ctx_base + i + 1 keys; 0: n_ctx_base */
    size_t n_items;    /* t * n_heads */
    int n_heads, n_kv_heads, head_dim, group;
    float scale;
    size_t next;       /* shared work counter */
    pthread_mutex_t mu;
} mt_job;

static void* mt_worker(void* arg) {
    mt_job* J = (mt_job*)arg;
    size_t hidden = (size_t)J->n_heads * J->head_dim;
    size_t max_ctx = J->n_ctx_base + (J->causal ? J->n_items / J->n_heads : 0) + 1;
    float* scores = (float*)malloc(sizeof(float) * max_ctx);
    if (!scores) return (void*)1;
    for (;;) {
        pthread_mutex_lock(&J->mu);
        size_t w = J->next;
        J->next += 8;
        pthread_mutex_unlock(&J->mu);
        if (w >= J->n_items) break;
        size_t wend = w + 8 < J->n_items ? w + 8 : J->n_items;
        for (; w < wend; ++w) {
            /* largest (latest) tokens first: they are the longest items */
            size_t item = J->n_items - 1 - w;
            size_t i = item / (size_t)J->n_heads;
            int h = (int)(item % (size_t)J->n_heads);
            size_t n_ctx = J->causal ? J->n_ctx_base + i + 1 : J->n_ctx_base;
            attend_head(J->q + i * hidden + (size_t)h * J->head_dim, J->k, J->v, n_ctx,
                        J->n_kv_heads, J->head_dim, h / J->group, J->scale, scores,
                        J->out + i * hidden + (size_t)h * J->head_dim);
        }
    }
    free(scores);
    return NULL;
}

static int run_mt(mt_job* J, int n_threads) {
    if (n_threads < 1) n_threads = 1;
    if (n_threads > 256) n_threads = 256;
    pthread_t th[256];
    J->next = 0;
    pthread_mutex_init(&J->mu, NULL);
    int started = 0, err = 0;
    for (int t = 0; t < n_threads; ++t) {
        if (pthread_create(&th[t], NULL, mt_worker, J) != 0) { err = -2; break; }
        ++started;
    }
    for (int t = 0; t < started; ++t) {
        void* r = NULL;
        pthread_join(th[t], &r);
        if (r) err = -2;
    }
    pthread_mutex_destroy(&J->mu);
    return err;
}

int orc_attention_decode_mt(const float* q, const float* k, const float* v, size_t n_ctx,
                            int n_heads, int n_kv_heads, int head_dim, float* out,
                            int n_threads) {
    if (n_heads <= 0 || n_kv_heads <= 0 || head_dim <= 0 || n_heads % n_kv_heads) return -1;
    mt_job J;
    memset(&J, 0, sizeof J);
    J.q = q; J.k = k; J.v = v; J.out = out;
    J.n_ctx_base = n_ctx; J.causal = 0; J.n_items = (size_t)n_heads;
    J.n_heads = n_heads; J.n_kv_heads = n_kv_heads; J.head_dim = head_dim;
    J.group = n_heads / n_kv_heads; J.scale = 1.0f / sqrtf((float)head_dim);
    return run_mt(&J, n_threads);
}

/* ------------------------------------------------------------ attn_batch --- */
/* Middle section of src/model.rs:232-254 (projections excluded): for each of the
 * t tokens, norm_rope_heads(q_i, pos0+i) and (k_i, pos0+i) in place; then for
 * each token append k_i, v_i to the cache (src/model.rs:241-242) and run
 * attention_decode over the n_ctx = cache_len keys now present (causal by
 * construction). cache_k/cache_v hold *cache_len rows of kv_dim floats and have
 * room for t more; *cache_len is advanced. out is [t][n_heads*head_dim].
 * n_threads > 1 is the harness extension: token-serial appends first, then the
 * (token, head) attention work spread over threads — identical arithmetic. */
int orc_attn_batch(float* q, float* k, const float* v, size_t t, size_t pos0,
                   const float* q_gain, const float* k_gain, float theta, float eps,
                   int n_heads, int n_kv_heads, int head_dim,
                   float* cache_k, float* cache_v, size_t* cache_len, float* out,
                   int n_threads) {
    if (n_heads <= 0 || n_kv_heads <= 0 || head_dim <= 0 || n_heads % n_kv_heads) return -1;
    size_t hidden = (size_t)n_heads * head_dim, kv_dim = (size_t)n_kv_heads * head_dim;
    for (size_t i = 0; i < t; ++i) {
        orc_norm_rope_heads(q + i * hidden, n_heads, head_dim, q_gain, pos0 + i, theta, eps);
        orc_norm_rope_heads(k + i * kv_dim, n_kv_heads, head_dim, k_gain, pos0 + i, theta, eps);
    }
    size_t base = *cache_len;
    if (n_threads <= 1) {
        for (size_t i = 0; i < t; ++i) {
            memcpy(cache_k + (base + i) * kv_dim, k + i * kv_dim, sizeof(float) * kv_dim);
            memcpy(cache_v + (base + i) * kv_dim, v + i * kv_dim, sizeof(float) * kv_dim);
            int rc = orc_attention_decode(q + i * hidden, cache_k, cache_v, base + i + 1,
                                          n_heads, n_kv_heads, head_dim, out + i * hidden);
            if (rc) return rc;
        }
    } else {
        memcpy(cache_k + base * kv_dim, k, sizeof(float) * kv_dim * t);
        memcpy(cache_v + base * kv_dim, v, sizeof(float) * kv_dim * t);
        mt_job J;
        memset(&J, 0, sizeof J);
        J.q = q; J.k = cache_k; J.v = cache_v; J.out = out;
        J.n_ctx_base = base; J.causal = 1; J.n_items = t * (size_t)n_heads;
        J.n_heads = n_heads; J.n_kv_heads = n_kv_heads; J.head_dim = head_dim;
        J.group = n_heads / n_kv_heads; J.scale = 1.0f / sqrtf((float)head_dim);
        int rc = run_mt(&J, n_threads);
        if (rc) return rc;
    }
    *cache_len = base + t;
    return 0;
}

/* ---------------------------------------------------------- attn_step --- */
/* Middle section of src/model.rs:440-451: norm+RoPE q (n_heads) and k
 * (n_kv_heads) at pos, append k, v, attend over every key in the window. */
int orc_attn_step(float* q, float* k, const float* v, size_t pos, const float* q_gain,
                  const float* k_gain, float theta, float eps, int n_heads, int n_kv_heads,
                  int head_dim, float* cache_k, float* cache_v, size_t* cache_len, float* out,
                  int n_threads) {
    size_t kv_dim = (size_t)n_kv_heads * head_dim;
    orc_norm_rope_heads(q, n_heads, head_dim, q_gain, pos, theta, eps);
    orc_norm_rope_heads(k, n_kv_heads, head_dim, k_gain, pos, theta, eps);
    memcpy(cache_k + *cache_len * kv_dim, k, sizeof(float) * kv_dim);
    memcpy(cache_v + *cache_len * kv_dim, v, sizeof(float) * kv_dim);
    *cache_len += 1;
    if (n_threads > 1)
        return orc_attention_decode_mt(q, cache_k, cache_v, *cache_len, n_heads, n_kv_heads,
                                       head_dim, out, n_threads);
    return orc_attention_decode(q, cache_k, cache_v, *cache_len, n_heads, n_kv_heads, head_dim,
                                out);
}

int orc_max_threads(void) {
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    return n > 0 ? (int)n : 1;
}
