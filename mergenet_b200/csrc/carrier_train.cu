// The carrier block's soft-top-k training terms (opentome/models/mergenet/
// model.py:1163-1206), forward and backward:
//
// * the straight-through carrier weights (model.py:1176-1179):
//   topk_x_trace * (1 + (w - w.detach())) with w = soft_sel gathered at the
//   carriers' patch indices.  The forward value is topk_x_trace itself; the
//   backward passes the gradient through and gives soft_sel, at each
//   carrier's patch, the dot product of the carrier's gradient and features.
// * the soft-top-k auxiliary representation (model.py:1196-1198):
//   aux[b] = sum_i x[b, i] * soft_sel[b, i] / max(sum_j soft_sel[b, j], 1e-6).
//
// All sums are fixed-order (no atomics): per channel over the rows in row
// order, per row over the channels in lane order then a warp tree.
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace mn {
namespace {

constexpr float kAuxEps = 1e-6f;  // the clamp of the soft weights' row sum

// Row sum of the soft weights (every thread gets it).  red: >= 32 floats.
__device__ __forceinline__ float weight_sum(const float* __restrict__ w, int n, float* red) {
  float s = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) s += w[i];
  return block_sum(s, red);
}

// aux[b, c]: grid (B, ceil(C / 128)), 256 threads.  Threads t and t + 128
// take the even and odd rows of channel c; the two partial sums are added in
// that order.
template <typename ET>
__global__ void __launch_bounds__(256) aux_forward_kernel(const ET* __restrict__ x, int64_t xb, int64_t xn, int n,
                                                          int C, const float* __restrict__ sel,
                                                          float* __restrict__ aux) {
  __shared__ float red[32];
  __shared__ float part[128];
  const int b = blockIdx.x;
  const float* w = sel + (int64_t)b * n;
  const float s = weight_sum(w, n, red);
  const float inv = 1.0f / fmaxf(s, kAuxEps);
  const int c = blockIdx.y * 128 + (threadIdx.x & 127);
  const int half = threadIdx.x >> 7;
  float acc = 0.f;
  if (c < C) {
    const ET* xr = x + (int64_t)b * xb + c;
    for (int i = half; i < n; i += 2) acc = fmaf(to_f32(xr[(int64_t)i * xn]), w[i] * inv, acc);
  }
  if (half == 1) part[threadIdx.x & 127] = acc;
  __syncthreads();
  if (half == 0 && c < C) aux[(int64_t)b * C + c] = acc + part[threadIdx.x];
}

// Backward of aux, part 1: one warp per row i of image b (grid (B,
// ceil(n / 8)), 256 threads).  grad_x[b, i, :] = wn_i * g[b, :] and
// dwn[b, i] = x[b, i, :] . g[b, :].
template <typename ET>
__global__ void __launch_bounds__(256) aux_backward_rows_kernel(const ET* __restrict__ x, int64_t xb, int64_t xn,
                                                                int n, int C, const float* __restrict__ sel,
                                                                const float* __restrict__ g,
                                                                ET* __restrict__ grad_x,
                                                                float* __restrict__ dwn) {
  __shared__ float red[32];
  const int b = blockIdx.x;
  const float* w = sel + (int64_t)b * n;
  const float s = weight_sum(w, n, red);
  const float inv = 1.0f / fmaxf(s, kAuxEps);
  const int lane = threadIdx.x & 31;
  const int i = blockIdx.y * 8 + (threadIdx.x >> 5);
  if (i >= n) return;
  const ET* xr = x + (int64_t)b * xb + (int64_t)i * xn;
  const float* gb = g + (int64_t)b * C;
  ET* gx = grad_x + ((int64_t)b * n + i) * C;
  const float wn = w[i] * inv;
  float dot = 0.f;
  for (int c = lane; c < C; c += 32) {
    const float gc = gb[c];
    dot = fmaf(to_f32(xr[c]), gc, dot);
    gx[c] = from_f32<ET>(wn * gc);
  }
  dot = warp_sum(dot);
  if (lane == 0) dwn[(int64_t)b * n + i] = dot;
}

// Backward of aux, part 2: one CTA per image.  wn = w / s' with
// s' = max(s, eps): dw_i = dwn_i / s' - [s > eps] (sum_j dwn_j w_j) / s'^2.
__global__ void __launch_bounds__(256) aux_backward_weights_kernel(int n, const float* __restrict__ sel,
                                                                   const float* __restrict__ dwn,
                                                                   float* __restrict__ grad_sel) {
  __shared__ float red[32];
  const int b = blockIdx.x;
  const float* w = sel + (int64_t)b * n;
  const float* d = dwn + (int64_t)b * n;
  const float s = weight_sum(w, n, red);
  float t = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) t = fmaf(d[i], w[i], t);
  t = block_sum(t, red);
  const float sp = fmaxf(s, kAuxEps);
  const float corr = s > kAuxEps ? t / (sp * sp) : 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) grad_sel[(int64_t)b * n + i] = d[i] / sp - corr;
}

// Straight-through weights, backward: one warp per carrier (b, j):
// grad_sel[b, idx[b, j]] = grad[b, j, :] . x[b, j, :].  grad_sel is zeroed
// first; a carrier index outside [0, n) is skipped and flagged.
template <typename ET>
__global__ void __launch_bounds__(256) ste_backward_kernel(const ET* __restrict__ x, int64_t xb, int64_t xk,
                                                           const ET* __restrict__ g, int64_t gb, int64_t gk,
                                                           const int64_t* __restrict__ idx, int B, int k, int C,
                                                           int n, float* __restrict__ grad_sel, int* status) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= (int64_t)B * k) return;
  const int b = (int)(row / k), j = (int)(row % k);
  const ET* xr = x + (int64_t)b * xb + (int64_t)j * xk;
  const ET* gr = g + (int64_t)b * gb + (int64_t)j * gk;
  float dot = 0.f;
  for (int c = lane; c < C; c += 32) dot = fmaf(to_f32(gr[c]), to_f32(xr[c]), dot);
  dot = warp_sum(dot);
  if (lane == 0) {
    const int64_t p = idx[(int64_t)b * k + j];
    if (p >= 0 && p < n) grad_sel[(int64_t)b * n + p] = dot;
    else if (status) atomicOr(status, MN_STATUS_TOO_MANY_EDGES);
  }
}

template <typename F>
int dispatch16(int dtype, F&& f) {
  if (dtype == MN_F32) { f(float{}); return MN_OK; }
  if (dtype == MN_F16) { f(__half{}); return MN_OK; }
  if (dtype == MN_BF16) { f(__nv_bfloat16{}); return MN_OK; }
  return MN_ERR_ARG;
}

int launch_status() { return cudaGetLastError() == cudaSuccess ? MN_OK : MN_ERR_LAUNCH; }

}  // namespace
}  // namespace mn

using namespace mn;

extern "C" int mn_soft_topk_aux(int batch, int n, int channels, int dtype, const void* x, int64_t x_batch_stride,
                                int64_t x_row_stride, const float* soft_sel, float* aux, void* stream) {
  if (batch < 0 || n <= 0 || channels <= 0) return MN_ERR_ARG;
  if (batch == 0) return MN_OK;
  if (!x || !soft_sel || !aux) return MN_ERR_ARG;
  cudaGetLastError();
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const dim3 grid((unsigned)batch, (unsigned)((channels + 127) / 128));
  const int rc = dispatch16(dtype, [&](auto tag) {
    using ET = decltype(tag);
    aux_forward_kernel<ET><<<grid, 256, 0, st>>>(static_cast<const ET*>(x), x_batch_stride, x_row_stride, n,
                                                 channels, soft_sel, aux);
  });
  return rc != MN_OK ? rc : launch_status();
}

extern "C" size_t mn_soft_topk_aux_backward_workspace_bytes(int batch, int n) {
  return batch > 0 && n > 0 ? (size_t)batch * n * sizeof(float) : 0;
}

extern "C" int mn_soft_topk_aux_backward(int batch, int n, int channels, int dtype, const void* x,
                                         int64_t x_batch_stride, int64_t x_row_stride, const float* soft_sel,
                                         const float* grad_aux, void* grad_x, float* grad_sel, void* workspace,
                                         size_t workspace_bytes, void* stream) {
  if (batch < 0 || n <= 0 || channels <= 0) return MN_ERR_ARG;
  if (batch == 0) return MN_OK;
  if (!x || !soft_sel || !grad_aux || !grad_x || !grad_sel || !workspace) return MN_ERR_ARG;
  if (workspace_bytes < mn_soft_topk_aux_backward_workspace_bytes(batch, n)) return MN_ERR_WORKSPACE;
  cudaGetLastError();
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  float* dwn = static_cast<float*>(workspace);
  const dim3 grid((unsigned)batch, (unsigned)((n + 7) / 8));
  const int rc = dispatch16(dtype, [&](auto tag) {
    using ET = decltype(tag);
    aux_backward_rows_kernel<ET><<<grid, 256, 0, st>>>(static_cast<const ET*>(x), x_batch_stride, x_row_stride, n,
                                                       channels, soft_sel, grad_aux, static_cast<ET*>(grad_x), dwn);
  });
  if (rc != MN_OK) return rc;
  aux_backward_weights_kernel<<<batch, 256, 0, st>>>(n, soft_sel, dwn, grad_sel);
  return launch_status();
}

extern "C" int mn_carrier_ste_backward(int batch, int k, int channels, int dtype, const void* topk_x,
                                       int64_t x_batch_stride, int64_t x_row_stride, const void* grad_out,
                                       int64_t g_batch_stride, int64_t g_row_stride, const int64_t* topk_idx,
                                       int n, float* grad_sel, int* status, void* stream) {
  if (batch < 0 || k < 0 || channels <= 0 || n <= 0 || !grad_sel) return MN_ERR_ARG;
  cudaGetLastError();
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaMemsetAsync(grad_sel, 0, (size_t)batch * n * sizeof(float), st);
  if ((int64_t)batch * k == 0) return launch_status();
  if (!topk_x || !grad_out || !topk_idx) return MN_ERR_ARG;
  const unsigned blocks = (unsigned)(((int64_t)batch * k + 7) / 8);
  const int rc = dispatch16(dtype, [&](auto tag) {
    using ET = decltype(tag);
    ste_backward_kernel<ET><<<blocks, 256, 0, st>>>(static_cast<const ET*>(topk_x), x_batch_stride, x_row_stride,
                                                    static_cast<const ET*>(grad_out), g_batch_stride, g_row_stride,
                                                    topk_idx, batch, k, channels, n, grad_sel, status);
  });
  return rc != MN_OK ? rc : launch_status();
}
