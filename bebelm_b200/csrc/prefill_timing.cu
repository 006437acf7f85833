// Timing and trace program for prefill_kernel (developer tool; not part of the library).
//
// Runs the kernel alone on t tokens of deterministic bf16 data (32 query heads, 8 kv heads,
// empty cache), 3 warm-up launches, then one launch timed with CUDA events:
//
//   nvcc -gencode arch=compute_100a,code=sm_100a -O3 -std=c++17 -DPLAIN \
//        bebelm_b200/csrc/prefill_timing.cu -o prefill_timing -lcuda && ./prefill_timing 8192
//
// Without -DPLAIN the kernel's clock64 trace points are compiled in (BEBELM_PREFILL_TRACE) and
// the program also prints, for the first CTA's first 17 key tiles, the cycle at which each
// hand-off happened (TMA issue, K landed, S issue, S seen by softmax, S fully read, P written,
// PV issue), relative to the first TMA issue.
#ifndef PLAIN
#define BEBELM_PREFILL_TRACE 1
#endif
#include "prefill.cu"
#include <cstdio>
#include <vector>
using namespace bebelm;
int main(int argc, char** argv) {
  int t = argc > 1 ? atoi(argv[1]) : 2048;
  int H = 32, KV = 8;
  size_t qn = (size_t)t * H * 64, kn = (size_t)t * KV * 64;
  std::vector<__nv_bfloat16> hq(qn), hk(kn);
  for (size_t i = 0; i < qn; ++i) hq[i] = __float2bfloat16((float)((i * 2654435761u) % 1000) / 1000.f - 0.5f);
  for (size_t i = 0; i < kn; ++i) hk[i] = __float2bfloat16((float)((i * 40503u) % 1000) / 1000.f - 0.5f);
  __nv_bfloat16 *q, *k, *v; float* out; int* err;
  cudaMalloc(&q, qn * 2); cudaMalloc(&k, kn * 2); cudaMalloc(&v, kn * 2); cudaMalloc(&out, qn * 4); cudaMalloc(&err, 4);
  cudaMemcpy(q, hq.data(), qn * 2, cudaMemcpyHostToDevice); cudaMemcpy(k, hk.data(), kn * 2, cudaMemcpyHostToDevice);
  cudaMemcpy(v, hk.data(), kn * 2, cudaMemcpyHostToDevice); cudaMemset(err, 0, 4);
  PrefillArgs a{}; a.q = q; a.k = k; a.v = v; a.out = out; a.t = t; a.len_before = 0; a.n_heads = H; a.n_kv = KV;
  a.scale_log2 = 0.18f; a.err = err;
  cudaEvent_t e0, e1; cudaEventCreate(&e0); cudaEventCreate(&e1);
  PrefillMaps mp; prefill_make_maps(a, &mp); for (int w = 0; w < 3; ++w) launch_prefill(a, mp, 0);
#ifndef PLAIN
  std::vector<long long> z(16 * 2 * 64, 0); cudaMemcpyToSymbol(g_trace, z.data(), z.size() * 8);
#endif
  cudaEventRecord(e0); launch_prefill(a, mp, 0); cudaEventRecord(e1); cudaEventSynchronize(e1);
  float ms; cudaEventElapsedTime(&ms, e0, e1);
  printf("t=%d kernel %.1f us  (%s)\n", t, ms * 1000, cudaGetErrorString(cudaGetLastError()));
#ifndef PLAIN
  std::vector<long long> tr(16 * 2 * 64); cudaMemcpyFromSymbol(tr.data(), g_trace, tr.size() * 8);
  const char* names[] = {"", "PV iss", "S iss", "S seen", "P done", "TMA", "p1 end", "p2 end", "st wait", "ld st", "ld dn", "S read", "K first", "PV start", "S start", "landed"};
  long long t0 = tr[(5 * 2 + 0) * 64 + 0];
  printf("%3s %2s", "j", "X");
  int evs[] = {5, 15, 12, 14, 2, 3, 11, 4, 13, 1};
  for (int ev : evs) printf(" %8s", names[ev]);
  printf("\n");
  for (int j = 0; j < 17; ++j) for (int X = 0; X < 2; ++X) {
    printf("%3d %2d", j, X);
    for (int ev : evs) { long long v = tr[(ev * 2 + (ev == 5 ? 0 : ev == 15 ? X : X)) * 64 + j]; printf(" %8lld", v ? v - t0 : -1); }
    printf("\n");
  }
#endif
  return 0;
}
