// The logits head and the greedy token choice on the device.
//
//   rmsnorm_row_kernel   final RMSNorm of a hidden state (src/kernels/rmsnorm.rs:10-21, used by
//                        logits_from_hidden, src/model.rs:379-388): Σ (x·x) widened to f64,
//                        mean = (f32)(ss / n), scale = 1 / sqrt(mean + eps), out = (x·scale)·g.
//                        One CTA; the f64 sum is a fixed tree (per-thread strided sums, then
//                        warp and CTA reductions), so it is deterministic, and equal to the
//                        reference's sequential sum whenever its partial sums are exact in f64.
//   mark_history_kernel  the presence set of Sampler::sample's repeat penalty
//                        (src/sampler.rs:66-84): a bitmap with one bit per token in `history`.
//   argmax_kernel        Sampler::sample with temperature <= 0 (src/sampler.rs:86-88, argmax
//                        :139-149): each token in the presence set once, l > 0 ? l / p : l · p,
//                        written back; then the first index of the maximum, scanning with a
//                        strict `>` from -inf (NaN never wins; all NaN / -inf gives 0).
// The logits themselves come from the quantized matvec of quant.cu (launch_qmv_multi).
#include <math_constants.h>

#include <algorithm>

#include "internal.h"

namespace bebelm {
namespace {

constexpr int kThreads = 1024;

__device__ __forceinline__ double warp_sum_f64(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__global__ void __launch_bounds__(kThreads) rmsnorm_row_kernel(const float* x, const float* gain, int n, float eps,
                                                               float* out) {
    __shared__ double part[kThreads / 32];
    __shared__ float s_scale;
    double ss = 0.0;
    for (int i = threadIdx.x; i < n; i += kThreads) ss += (double)__fmul_rn(x[i], x[i]);
    ss = warp_sum_f64(ss);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
        double v = part[threadIdx.x];
        v = warp_sum_f64(v);
        if (threadIdx.x == 0) {
            const float mean = __double2float_rn(v / (double)n);
            s_scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
        }
    }
    __syncthreads();
    const float scale = s_scale;
    for (int i = threadIdx.x; i < n; i += kThreads) out[i] = __fmul_rn(__fmul_rn(x[i], scale), gain[i]);
}

__global__ void mark_history_kernel(const uint32_t* history, size_t n_history, size_t n, uint32_t* bitmap) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_history; i += (size_t)gridDim.x * blockDim.x) {
        const uint32_t t = history[i];
        if (t < n) atomicOr(bitmap + (t >> 5), 1u << (t & 31));  // out-of-range ids are ignored
    }
}

struct Best {
    float v;
    uint32_t i;  // 0xffffffff: none yet
};
// a before b in the reference's scan: a value above every earlier one, first index on ties
__device__ __forceinline__ Best better(Best a, Best b) {
    if (a.i == 0xffffffffu) return b;
    if (b.i == 0xffffffffu) return a;
    if (a.v > b.v || (a.v == b.v && a.i < b.i)) return a;
    return b;
}

__global__ void __launch_bounds__(kThreads) argmax_kernel(float* x, size_t n, const uint32_t* bitmap, float penalty,
                                                          uint32_t* out) {
    __shared__ Best part[kThreads / 32];
    Best best{-CUDART_INF_F, 0xffffffffu};
    for (size_t i = threadIdx.x; i < n; i += kThreads) {
        float v = x[i];
        if (bitmap && ((bitmap[i >> 5] >> (i & 31)) & 1u)) {
            v = v > 0.0f ? __fdiv_rn(v, penalty) : __fmul_rn(v, penalty);
            x[i] = v;
        }
        if (v > best.v) best = Best{v, (uint32_t)i};  // strict: a thread's first index of its max
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const Best other{__shfl_xor_sync(0xffffffffu, best.v, o), __shfl_xor_sync(0xffffffffu, best.i, o)};
        best = better(best, other);
    }
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x < 32) {
        best = part[threadIdx.x];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const Best other{__shfl_xor_sync(0xffffffffu, best.v, o), __shfl_xor_sync(0xffffffffu, best.i, o)};
            best = better(best, other);
        }
        if (threadIdx.x == 0) *out = best.i == 0xffffffffu ? 0u : best.i;
    }
}

}  // namespace

cudaError_t launch_rmsnorm_row(const float* x, const float* gain, int n, float eps, float* out, cudaStream_t s) {
    rmsnorm_row_kernel<<<1, kThreads, 0, s>>>(x, gain, n, eps, out);
    return cudaGetLastError();
}

cudaError_t launch_greedy(float* logits, size_t n, const uint32_t* history, size_t n_history, float penalty,
                          uint32_t* bitmap, uint32_t* token, cudaStream_t s) {
    const bool pen = penalty != 1.0f && n_history > 0;
    if (pen) {
        cudaError_t e = cudaMemsetAsync(bitmap, 0, (n + 31) / 32 * 4, s);
        if (e != cudaSuccess) return e;
        const unsigned blocks = (unsigned)std::min<size_t>((n_history + 255) / 256, 148);
        mark_history_kernel<<<blocks, 256, 0, s>>>(history, n_history, n, bitmap);
    }
    argmax_kernel<<<1, kThreads, 0, s>>>(logits, n, pen ? bitmap : nullptr, penalty, token);
    return cudaGetLastError();
}

}  // namespace bebelm
