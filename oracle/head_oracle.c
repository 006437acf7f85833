/*
 * CPU oracle, greedy token choice (TEST INFRASTRUCTURE ONLY: the product never links this).
 *
 * Restates, in plain C:
 *   argmax                    src/sampler.rs:139-149: strict `>` scan from -inf, best starts
 *                             at 0 (first index of the maximum; NaN never wins)
 *   Sampler::sample, greedy   src/sampler.rs:64-88 with temperature <= 0: when the repeat
 *                             penalty is not 1, each distinct token of `history` once:
 *                             l > 0 ? l / p : l * p (logits rewritten in place), then argmax
 * Pinned by the reference's sampler tests (src/sampler.rs:154-187, transcribed in
 * tests/golden). The logits head (src/model.rs:379-388) composes orc_rmsnorm and orc_matvec.
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <stdlib.h>

size_t orc_argmax(const float* x, size_t n) {
    size_t best = 0;
    float best_v = -INFINITY;
    for (size_t i = 0; i < n; ++i)
        if (x[i] > best_v) {
            best_v = x[i];
            best = i;
        }
    return best;
}

/* 0 on success, -1 for a history id out of range (the reference indexes out of bounds). */
int orc_sample_greedy(float* logits, size_t n, const uint32_t* history, size_t n_history, float penalty,
                      uint32_t* token) {
    if (penalty != 1.0f) {
        unsigned char* seen = calloc(n ? n : 1, 1);
        if (!seen) return -1;
        for (size_t i = 0; i < n_history; ++i) {
            const uint32_t t = history[i];
            if (t >= n) {
                free(seen);
                return -1;
            }
            if (!seen[t]) {
                seen[t] = 1;
                logits[t] = logits[t] > 0.0f ? logits[t] / penalty : logits[t] * penalty;
            }
        }
        free(seen);
    }
    *token = (uint32_t)orc_argmax(logits, n);
    return 0;
}
