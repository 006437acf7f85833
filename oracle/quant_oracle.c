/*
 * CPU oracle, quantized part (TEST INFRASTRUCTURE ONLY: the product never links this).
 *
 * Restates, in plain C, the reference's GGML dequantization and quantized matrix-vector
 * product, the arithmetic that feeds the attention path's q/k/v/o projections:
 *   f16_to_f32                src/kernels/dequant.rs:22-54
 *   get_scale_min_k4          src/kernels/dequant.rs:64-73
 *   dequantize_q4_k_block     src/kernels/dequant.rs:75-109
 *   dequantize_q6_k_block     src/kernels/dequant.rs:112-140
 *   dequantize_into           src/kernels/dequant.rs:151-176
 *   quantize_q8               src/kernels/matmul.rs:141-164
 *   dot_q4k_block_q8          src/kernels/matmul.rs:220-244 (exact i32 sub-block dots)
 *   dot_q6k_block_q8          src/kernels/matmul.rs:633-646, q6k_block_idot_portable :650-700
 *   dot_q{4,6}k_row_q8        src/kernels/matmul.rs:293-300, 748-754 (sequential f32 sum)
 *   matvec                    src/kernels/matmul.rs:850-905
 *   matmul                    src/kernels/matmul.rs:908-1013 (bit-identical to matvec per token)
 * Compiled with -ffp-contract=off: every f32 product and sum rounds once, as in the Rust.
 * The integer parts are exact, so for Q4_K/Q6_K weights the result is the reference's bit for
 * bit (pinned by the reference's own unit tests, transcribed in tests/golden). F32/F16 weights go
 * through `dot`, whose final lane reduction order is not visible (see orc_dot).
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>

float orc_dot(const float* a, const float* b, size_t n);

enum { GG_F32 = 0, GG_F16 = 1, GG_Q4_K = 12, GG_Q6_K = 14 };
#define QK_K 256
#define Q4K_BYTES 144
#define Q6K_BYTES 210

float orc_f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t exp = (h >> 10) & 0x1fu, mant = h & 0x03ffu;
    uint32_t bits;
    if (exp == 0) {
        if (mant == 0) {
            bits = sign;
        } else {  // subnormal: normalise into an f32 normal
            int e = -1;
            uint32_t m = mant;
            do {
                ++e;
                m <<= 1;
            } while (!(m & 0x0400u));
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | ((m & 0x03ffu) << 13);
        }
    } else if (exp == 0x1f) {
        bits = sign | 0x7f800000u | (mant << 13);
    } else {
        bits = sign | ((exp - 15 + 127) << 23) | (mant << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static float rd_f16(const uint8_t* p) { return orc_f16_to_f32((uint16_t)(p[0] | (p[1] << 8))); }

static void scale_min_k4(int j, const uint8_t* s, uint8_t* sc, uint8_t* m) {
    if (j < 4) {
        *sc = s[j] & 63;
        *m = s[j + 4] & 63;
    } else {
        *sc = (uint8_t)((s[j + 4] & 0x0f) | ((s[j - 4] >> 6) << 4));
        *m = (uint8_t)((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
    }
}

static void deq_q4k(const uint8_t* b, float* out) {
    const float d = rd_f16(b), dmin = rd_f16(b + 2);
    const uint8_t *scales = b + 4, *qs = b + 16;
    int oi = 0;
    for (int chunk = 0; chunk < 4; ++chunk) {
        uint8_t sc1, m1, sc2, m2;
        scale_min_k4(2 * chunk, scales, &sc1, &m1);
        scale_min_k4(2 * chunk + 1, scales, &sc2, &m2);
        const float d1 = d * (float)sc1, mn1 = dmin * (float)m1, d2 = d * (float)sc2, mn2 = dmin * (float)m2;
        const uint8_t* q = qs + chunk * 32;
        for (int i = 0; i < 32; ++i) out[oi++] = d1 * (float)(q[i] & 0x0f) - mn1;
        for (int i = 0; i < 32; ++i) out[oi++] = d2 * (float)(q[i] >> 4) - mn2;
    }
}

static void deq_q6k(const uint8_t* b, float* out) {
    const float d = rd_f16(b + 208);
    for (int n = 0; n < 2; ++n) {
        const uint8_t *ql = b + n * 64, *qh = b + 128 + n * 32;
        const int8_t* sc = (const int8_t*)(b + 192 + n * 8);
        float* o = out + n * 128;
        for (int l = 0; l < 32; ++l) {
            const int is = l / 16;
            const int q1 = ((ql[l] & 0x0f) | (((qh[l] >> 0) & 3) << 4)) - 32;
            const int q2 = ((ql[l + 32] & 0x0f) | (((qh[l] >> 2) & 3) << 4)) - 32;
            const int q3 = ((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
            const int q4 = ((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
            o[l] = d * (float)sc[is] * (float)q1;
            o[l + 32] = d * (float)sc[is + 2] * (float)q2;
            o[l + 64] = d * (float)sc[is + 4] * (float)q3;
            o[l + 96] = d * (float)sc[is + 6] * (float)q4;
        }
    }
}

/* n elements of `dtype` from `data` into out; -1 for an unsupported dtype or a partial block */
int orc_dequantize(int dtype, const uint8_t* data, size_t n, float* out) {
    switch (dtype) {
        case GG_F32:
            memcpy(out, data, 4 * n);
            return 0;
        case GG_F16:
            for (size_t i = 0; i < n; ++i) out[i] = rd_f16(data + 2 * i);
            return 0;
        case GG_Q4_K:
            if (n % QK_K) return -1;
            for (size_t b = 0; b < n / QK_K; ++b) deq_q4k(data + b * Q4K_BYTES, out + b * QK_K);
            return 0;
        case GG_Q6_K:
            if (n % QK_K) return -1;
            for (size_t b = 0; b < n / QK_K; ++b) deq_q6k(data + b * Q6K_BYTES, out + b * QK_K);
            return 0;
        default:
            return -1;
    }
}

/* quantize_q8: per 256-block scale = max|x| / 127, q = round(x * 127/max|x|) (half away from
 * zero, as Rust's f32::round) clamped to +-127, and the sum of each 32-wide sub-block's quants */
void orc_quantize_q8(const float* x, size_t n, int8_t* q, float* scales, int32_t* sums) {
    for (size_t b = 0; b < n / QK_K; ++b) {
        const float* xb = x + b * QK_K;
        float amax = 0.0f;
        for (int i = 0; i < QK_K; ++i) amax = fmaxf(amax, fabsf(xb[i]));
        scales[b] = amax / 127.0f;
        const float inv = amax > 0.0f ? 127.0f / amax : 0.0f;
        int8_t* qb = q + b * QK_K;
        for (int i = 0; i < QK_K; ++i) {
            float r = roundf(xb[i] * inv);
            if (r < -127.0f) r = -127.0f;
            if (r > 127.0f) r = 127.0f;
            qb[i] = (int8_t)r;
        }
        for (int s = 0; s < 8; ++s) {
            int32_t t = 0;
            for (int i = 0; i < 32; ++i) t += qb[s * 32 + i];
            sums[b * 8 + s] = t;
        }
    }
}

static float dot_q4k_block_q8(const uint8_t* blk, const int8_t* qx, float sx, const int32_t* sums) {
    const float d = rd_f16(blk), dmin = rd_f16(blk + 2);
    const uint8_t *scales = blk + 4, *qs = blk + 16;
    int32_t sc[8], sm = 0, sd = 0;
    for (int j = 0; j < 8; ++j) {
        uint8_t s, m;
        scale_min_k4(j, scales, &s, &m);
        sc[j] = s;
        sm += (int32_t)m * sums[j];
    }
    for (int c = 0; c < 4; ++c) {
        int32_t lo = 0, hi = 0;
        for (int i = 0; i < 32; ++i) {
            lo += (int32_t)(qs[c * 32 + i] & 0x0f) * qx[(2 * c) * 32 + i];
            hi += (int32_t)(qs[c * 32 + i] >> 4) * qx[(2 * c + 1) * 32 + i];
        }
        sd += sc[2 * c] * lo + sc[2 * c + 1] * hi;
    }
    return sx * (d * (float)sd - dmin * (float)sm);
}

static float dot_q6k_block_q8(const uint8_t* blk, const int8_t* qx, float sx) {
    const float d = rd_f16(blk + 208);
    int32_t s = 0;
    for (int n = 0; n < 2; ++n) {
        const uint8_t *ql = blk + n * 64, *qh = blk + 128 + n * 32;
        const int8_t* sc = (const int8_t*)(blk + 192 + n * 8);
        /* groups: (ql offset within the half, high nibble?, qh shift); 2 x 16-wide sub-blocks each */
        static const int off[4] = {0, 32, 0, 32}, high[4] = {0, 0, 1, 1}, sh[4] = {0, 2, 4, 6};
        for (int g = 0; g < 4; ++g)
            for (int sub = 0; sub < 2; ++sub) {
                const int k = n * 8 + 2 * g + sub;
                int32_t t = 0;
                for (int i = 0; i < 16; ++i) {
                    const uint8_t l = ql[off[g] + sub * 16 + i];
                    const int nib = high[g] ? (l >> 4) & 0x0f : l & 0x0f;
                    const int h = (qh[sub * 16 + i] >> sh[g]) & 3;
                    t += ((nib | (h << 4)) - 32) * qx[k * 16 + i];
                }
                s += t * (int32_t)sc[2 * g + sub];
            }
    }
    return sx * (d * (float)s);
}

/* y[n_out] = W x, W [n_out rows][n_in] packed as dtype (row-major by output). 0 or -1. */
int orc_matvec(int dtype, const uint8_t* w, size_t n_in, size_t n_out, const float* x, float* y, float* scratch,
               int8_t* q8, float* q8_scales, int32_t* q8_sums) {
    if (dtype == GG_Q4_K || dtype == GG_Q6_K) {
        if (n_in % QK_K) return -1;
        orc_quantize_q8(x, n_in, q8, q8_scales, q8_sums);
        const size_t nb = n_in / QK_K, bb = dtype == GG_Q4_K ? Q4K_BYTES : Q6K_BYTES;
        for (size_t o = 0; o < n_out; ++o) {
            const uint8_t* row = w + o * nb * bb;
            float acc = -0.0f; /* Iterator::sum over f32, in block order */
            for (size_t b = 0; b < nb; ++b)
                acc += dtype == GG_Q4_K
                           ? dot_q4k_block_q8(row + b * bb, q8 + b * QK_K, q8_scales[b], q8_sums + b * 8)
                           : dot_q6k_block_q8(row + b * bb, q8 + b * QK_K, q8_scales[b]);
            y[o] = acc;
        }
        return 0;
    }
    if (dtype != GG_F32 && dtype != GG_F16) return -1;
    const size_t rb = (dtype == GG_F32 ? 4 : 2) * n_in;
    for (size_t o = 0; o < n_out; ++o) {
        orc_dequantize(dtype, w + o * rb, n_in, scratch);
        y[o] = orc_dot(scratch, x, n_in);
    }
    return 0;
}

/* Y = W X for n_tokens token-major columns: per token exactly matvec (the reference's batched
 * kernels are bit-identical to it). */
int orc_matmul(int dtype, const uint8_t* w, size_t n_in, size_t n_out, const float* x, size_t n_tokens, float* y,
               float* scratch, int8_t* q8, float* q8_scales, int32_t* q8_sums) {
    for (size_t t = 0; t < n_tokens; ++t)
        if (orc_matvec(dtype, w, n_in, n_out, x + t * n_in, y + t * n_out, scratch, q8, q8_scales, q8_sums))
            return -1;
    return 0;
}
