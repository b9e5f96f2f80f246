// Threshold soft top-k of one row, executed by one thread block.
//
// Restates opentome/utils/thetopk.py:4-43 for a row whose values have already
// been scaled by the batch-global range (x / (max - min) * temperature).
// The two log-cum-sum-exp scans are accumulated in float64 and rounded to
// float32 per element, as the reference's CPU kernel does; everything after
// them (sqrt/exp/log threshold, bracket search, two-sided map) is float32 in
// the reference's operation order.
#pragma once

#include <climits>
#include <type_traits>

#include "common.cuh"

namespace mn {

struct RowScratch {
  float* xs;       // [np] sorted values (+inf padding)
  float* lse1;     // [np]
  float* xlamb;    // [np]
  double* dbuf;    // [np]
  double* dscr;    // [32]
  int* iscr;       // [32]
};

__host__ __device__ inline size_t row_scratch_bytes(int np) {
  return (size_t)np * (3 * sizeof(float) + sizeof(double)) + 32 * sizeof(double) + 32 * sizeof(int);
}

// Carve RowScratch out of a shared-memory region (8-byte aligned base).
__device__ __forceinline__ RowScratch carve_row_scratch(unsigned char* base, int np) {
  RowScratch r;
  r.dbuf = reinterpret_cast<double*>(base);
  r.dscr = r.dbuf + np;
  r.xs = reinterpret_cast<float*>(r.dscr + 32);
  r.lse1 = r.xs + np;
  r.xlamb = r.lse1 + np;
  r.iscr = reinterpret_cast<int*>(r.xlamb + np);
  return r;
}

// x: the n scaled values of this row, readable by every thread (shared or
// global).  Returns lambda in every thread.  np = next_pow2(n) and the block
// size must divide np (np >= blockDim.x) or be larger than np.
// *bracket (when given) receives the chosen bracket b: lambda = xlamb[b].
// The scratch keeps the sorted row (xs), lse1 and the suffix sums (dbuf)
// after the call, for the gradient.
__device__ __noinline__ static float thre_topk_lambda(const float* x, int n, int np, int k, RowScratch s,
                                                      int* bracket = nullptr) {
  const int tid = threadIdx.x;
  const int per_thread = np / (int)blockDim.x;
  if (np % (int)blockDim.x == 0 && (per_thread == 1 || per_thread == 2 || per_thread == 4) && blockDim.x >= 32) {
    // keys in registers, exchanged by shuffles and (for partners 32 .. blockDim
    // apart) through the scan buffer, which is free until the scans
    float* xb = reinterpret_cast<float*>(s.dbuf);
    auto run = [&](auto tag) {
      constexpr int R = decltype(tag)::value;
      float kv[R];
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const int i = tid + r * blockDim.x;
        kv[r] = (i < n) ? x[i] : INFINITY;
      }
      bitonic_sort_regs<R>(kv, xb, np);
#pragma unroll
      for (int r = 0; r < R; ++r) s.xs[tid + r * blockDim.x] = kv[r];
    };
    if (per_thread == 1) run(std::integral_constant<int, 1>{});
    else if (per_thread == 2) run(std::integral_constant<int, 2>{});
    else run(std::integral_constant<int, 4>{});
    __syncthreads();
  } else {
    for (int i = tid; i < np; i += blockDim.x) s.xs[i] = (i < n) ? x[i] : INFINITY;
    __syncthreads();
    bitonic_sort_f32(s.xs, np);
  }
  const double xmax = (double)s.xs[n - 1];
  const double xmin = (double)s.xs[0];
  // per-thread chunk for the scans
  const int per = (np + blockDim.x - 1) / blockDim.x;
  const int span = per * blockDim.x;  // >= np; dbuf sized np, so guard
  // ---- lse1[j] = log(sum_{i<=j} exp(xs_i)), offset by the row maximum
  for (int i = tid; i < np; i += blockDim.x) s.dbuf[i] = (i < n) ? exp((double)s.xs[i] - xmax) : 0.0;
  __syncthreads();
  if (span == np) {
    block_scan_inclusive(s.dbuf, per, s.dscr);
  } else {  // np < blockDim.x: serial-free fallback with per = 1 over the first np threads
    // (np < blockDim.x only for tiny rows; scan by thread 0)
    if (tid == 0) { double r = 0; for (int i = 0; i < np; ++i) { r += s.dbuf[i]; s.dbuf[i] = r; } }
    __syncthreads();
  }
  for (int i = tid; i < n; i += blockDim.x) s.lse1[i] = (float)(xmax + log(s.dbuf[i]));
  __syncthreads();
  // ---- suffix sums Q_i = sum_{i'>=i} exp(xmin - xs_i'), scanned in reverse
  for (int r = tid; r < np; r += blockDim.x) {
    int i = n - 1 - r;
    s.dbuf[r] = (i >= 0) ? exp(xmin - (double)s.xs[i]) : 0.0;
  }
  __syncthreads();
  if (span == np) {
    block_scan_inclusive(s.dbuf, per, s.dscr);
  } else {
    if (tid == 0) { double r = 0; for (int i = 0; i < np; ++i) { r += s.dbuf[i]; s.dbuf[i] = r; } }
    __syncthreads();
  }
  // ---- threshold candidates and the first bracket that holds
  int cand = INT_MAX;
  for (int j = tid; j < n; j += blockDim.x) {
    float lse2 = (j + 1 < n) ? (float)(-xmin + log(s.dbuf[n - 2 - j])) : -INFINITY;
    float l1 = s.lse1[j];
    int km = k - (n - 1 - j);
    float les = l1 + lse2;
    float term = sqrtf((float)((long long)km * km) + expf(les)) + (float)km;
    float xl = l1 - logf(fabsf(term) + 1e-8f);
    s.xlamb[j] = xl;
    float hi = (j + 1 < n) ? s.xs[j + 1] : INFINITY;
    if (xl >= s.xs[j] && xl <= hi) cand = min(cand, j);
  }
  int idx = block_min_int(cand, s.iscr);
  if (idx == INT_MAX) idx = 0;
  if (bracket) *bracket = idx;
  float lam = s.xlamb[idx];
  __syncthreads();
  return lam;
}

__device__ __forceinline__ float thre_topk_map(float x, float lam) {
  float delta = x - lam;
  return delta > 0.f ? 1.0f - 0.5f * expf(-delta) : 0.5f * expf(delta);
}

}  // namespace mn
