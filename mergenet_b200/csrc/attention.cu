// Sliding-window attention over the flattened token sequence with an optional
// per-key bias and a global CLS row, replacing the FlashAttention calls of
// unbiased_local_attention / biased_local_attention
// (opentome/timm/bias_local_attn.py:486-625, :243-483) and the CLS-row SDPA
// of LocalAttention.forward (:704-719).
//
// This file holds the CUDA-core path: one warp per query row with an online
// softmax over 32-key chunks, keys/values of the CTA's band staged in fp32
// shared memory.  Scores, softmax and the P.V accumulation are fp32.
#include <algorithm>

#include "common.cuh"

namespace mn {

bool attention_tc(int dtype, const void* q, int64_t qb, int64_t qn, int64_t qh, const void* k, const void* v,
                  int64_t kb, int64_t kn, int64_t kh, int B, int Nq, int Nk, int H, int D, int window, float scale,
                  const void* bias, int bias_dtype, void* out, int out_dtype, int* err, cudaStream_t st,
                  bool cls_global, bool* cls_done);

constexpr int kLocalQT = 32;  // queries per CTA

template <typename ET>
__global__ void __launch_bounds__(256) local_attn_kernel(
    const ET* __restrict__ q, const ET* __restrict__ k, const ET* __restrict__ v, int64_t sb, int64_t sn,
    int64_t sh, int N, int H, int D, const void* __restrict__ bias, int bias_dtype, int window, float scale,
    void* __restrict__ out, int out_dtype, int skip_row0) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int q0 = blockIdx.x * kLocalQT;
  const int h = blockIdx.y, b = blockIdx.z;
  const int W = window < 0 ? N : window;
  const int lo = max(0, q0 - W), hi = min(N, q0 + kLocalQT + W);
  const int nk = hi - lo;
  const int DS = D + 1;  // padded row stride (floats)
  float* ks = reinterpret_cast<float*>(smem_raw);  // [nk][DS]
  float* vs = ks + (size_t)nk * DS;                // [nk][DS]
  float* bs = vs + (size_t)nk * DS;                // [nk]
  float* qs = bs + nk;                             // [8 warps][D]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int64_t base = (int64_t)b * sb + (int64_t)h * sh;
  for (int i = threadIdx.x; i < nk * D; i += blockDim.x) {
    const int r = i / D, c = i % D;
    const int64_t off = base + (int64_t)(lo + r) * sn + c;
    ks[r * DS + c] = to_f32(k[off]);
    vs[r * DS + c] = to_f32(v[off]);
  }
  for (int r = threadIdx.x; r < nk; r += blockDim.x) {
    // the reference rounds the bias to the q/k/v dtype before use
    float bv = 0.f;
    if (bias) bv = to_f32(from_f32<ET>(load_any(bias, bias_dtype, (int64_t)b * N + lo + r)));
    bs[r] = bv;
  }
  __syncthreads();
  float* qw = qs + warp * D;
  for (int qi = q0 + warp; qi < min(N, q0 + kLocalQT); qi += nw) {
    if (skip_row0 && qi == 0) continue;
    const int64_t qoff = base + (int64_t)qi * sn;
    for (int c = lane; c < D; c += 32) qw[c] = to_f32(q[qoff + c]);
    __syncwarp();
    const int j0 = max(0, qi - W), j1 = min(N - 1, qi + W);
    float m = -INFINITY, l = 0.f;
    float o[4] = {0.f, 0.f, 0.f, 0.f};  // channels lane, lane+32, lane+64, lane+96
    for (int jc = j0; jc <= j1; jc += 32) {
      const int j = jc + lane;
      float s = -INFINITY;
      if (j <= j1) {
        const float* kr = ks + (j - lo) * DS;
        float acc = 0.f;
        for (int c = 0; c < D; ++c) acc = fmaf(qw[c], kr[c], acc);
        s = acc * scale + bs[j - lo];
      }
      const float mc = warp_max(s);
      const float mn = fmaxf(m, mc);
      const float p = (j <= j1) ? expf(s - mn) : 0.f;
      const float corr = (m == -INFINITY) ? 0.f : expf(m - mn);
      l = l * corr + warp_sum(p);
#pragma unroll
      for (int t = 0; t < 4; ++t) o[t] *= corr;
      const int cnt = min(32, j1 - jc + 1);
      for (int u = 0; u < cnt; ++u) {
        const float pu = __shfl_sync(MN_FULL_MASK, p, u);
        const float* vr = vs + (jc + u - lo) * DS;
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const int c = lane + 32 * t;
          if (c < D) o[t] = fmaf(pu, vr[c], o[t]);
        }
      }
      m = mn;
    }
    const float inv = 1.0f / l;
    const int64_t ooff = (((int64_t)b * N + qi) * H + h) * D;
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const int c = lane + 32 * t;
      if (c < D) store_any(out, out_dtype, ooff + c, o[t] * inv);
    }
    __syncwarp();
  }
}

// Row 0 (CLS) attends to every key: one CTA per (head, image).
template <typename ET>
__global__ void __launch_bounds__(256) cls_row_kernel(const ET* __restrict__ q, const ET* __restrict__ k,
                                                      const ET* __restrict__ v, int64_t sb, int64_t sn,
                                                      int64_t sh, int N, int H, int D,
                                                      const void* __restrict__ bias, int bias_dtype, float scale,
                                                      void* __restrict__ out, int out_dtype) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  float* p = reinterpret_cast<float*>(smem_raw);  // [N]
  float* qv = p + N;                              // [D]
  float* part = qv + D;                           // [256 * 8]
  __shared__ float red[64];
  const int h = blockIdx.x, b = blockIdx.y;
  const int64_t base = (int64_t)b * sb + (int64_t)h * sh;
  for (int c = threadIdx.x; c < D; c += blockDim.x) qv[c] = to_f32(q[base + c]);
  __syncthreads();
  float mx = -INFINITY, dummy = INFINITY;
  const bool vec = (D % 8 == 0) && (sn % 8 == 0) && ((reinterpret_cast<uintptr_t>(k + base) & 15) == 0);
  for (int j = threadIdx.x; j < N; j += blockDim.x) {
    const ET* kr = k + base + (int64_t)j * sn;
    float acc = 0.f;
    if (vec) {
      for (int c = 0; c < D; c += 8) {
        const uint4 u = *reinterpret_cast<const uint4*>(kr + c);
        const ET* e = reinterpret_cast<const ET*>(&u);
#pragma unroll
        for (int i = 0; i < 8; ++i) acc = fmaf(qv[c + i], to_f32(e[i]), acc);
      }
    } else {
      for (int c = 0; c < D; ++c) acc = fmaf(qv[c], to_f32(kr[c]), acc);
    }
    float s = acc * scale;
    if (bias) s += to_f32(from_f32<ET>(load_any(bias, bias_dtype, (int64_t)b * N + j)));
    p[j] = s;
    mx = fmaxf(mx, s);
  }
  block_minmax(dummy, mx, red);
  float sum = 0.f;
  for (int j = threadIdx.x; j < N; j += blockDim.x) {
    const float e = expf(p[j] - mx);
    p[j] = e;
    sum += e;
  }
  // block sum through the same scratch
  sum = warp_sum(sum);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sum;
  __syncthreads();
  float tot = 0.f;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) tot += red[w];
  __syncthreads();
  // o = sum_j p_j v_j: with 16-byte rows, D / 8 threads cover a value row
  // (8 channels each) and blockDim * 8 / D rows are summed in parallel, each
  // group keeping its own partial sums, combined at the end
  const bool vvec = vec && ((reinterpret_cast<uintptr_t>(v + base) & 15) == 0) && D <= 256;
  if (vvec) {
    const int per_row = D / 8;
    const int sub = threadIdx.x % per_row, rg = threadIdx.x / per_row, nrg = blockDim.x / per_row;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (rg < nrg)
      for (int j = rg; j < N; j += nrg) {
        const uint4 u = *reinterpret_cast<const uint4*>(v + base + (int64_t)j * sn + sub * 8);
        const ET* e = reinterpret_cast<const ET*>(&u);
        const float pj = p[j];
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] = fmaf(pj, to_f32(e[i]), acc[i]);
      }
    if (rg < nrg)
#pragma unroll
      for (int i = 0; i < 8; ++i) part[rg * D + sub * 8 + i] = acc[i];
    __syncthreads();
    for (int c = threadIdx.x; c < D; c += blockDim.x) {
      float o = 0.f;
      for (int gg = 0; gg < nrg; ++gg) o += part[gg * D + c];
      store_any(out, out_dtype, (((int64_t)b * N) * H + h) * D + c, o / tot);
    }
    return;
  }
  const int groups = blockDim.x / D > 0 ? blockDim.x / D : 1;
  const int c = threadIdx.x % D, g = threadIdx.x / D;
  float acc = 0.f;
  if (g < groups)
    for (int j = g; j < N; j += groups) acc = fmaf(p[j], to_f32(v[base + (int64_t)j * sn + c]), acc);
  part[threadIdx.x] = acc;
  __syncthreads();
  if (threadIdx.x < D) {
    float o = 0.f;
    for (int gg = 0; gg < groups; ++gg) o += part[gg * D + threadIdx.x];
    store_any(out, out_dtype, (((int64_t)b * N) * H + h) * D + threadIdx.x, o / tot);
  }
}

// General attention with separate query / key sequences (the recovery
// cross-attention, model.py:173-188: 393 carrier queries over 785 tokens) or
// a window.  Keys are streamed through shared memory in chunks of 64 with an
// online softmax; one warp owns 4 query rows.
constexpr int kXQ = 32;     // queries per CTA
constexpr int kXK = 64;     // keys per chunk
template <typename ET>
__global__ void __launch_bounds__(256) attn_chunked_kernel(
    const ET* __restrict__ q, int64_t qb, int64_t qn, int64_t qh, const ET* __restrict__ k,
    const ET* __restrict__ v, int64_t kb, int64_t kn, int64_t kh, int Nq, int Nk, int H, int D, int window,
    float scale, void* __restrict__ out, int out_dtype) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int DS = D + 1;
  float* qs = reinterpret_cast<float*>(smem_raw);  // [kXQ][D]
  float* ks = qs + kXQ * D;                        // [kXK][DS]
  float* vs = ks + kXK * DS;                       // [kXK][DS]
  const int q0 = blockIdx.x * kXQ, h = blockIdx.y, b = blockIdx.z;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t qbase = (int64_t)b * qb + (int64_t)h * qh;
  const int64_t kbase = (int64_t)b * kb + (int64_t)h * kh;
  for (int i = threadIdx.x; i < kXQ * D; i += blockDim.x) {
    const int r = i / D, c = i % D;
    qs[i] = (q0 + r < Nq) ? to_f32(q[qbase + (int64_t)(q0 + r) * qn + c]) : 0.f;
  }
  int lo = 0, hi = Nk;
  if (window >= 0) {
    lo = max(0, q0 - window);
    hi = min(Nk, q0 + kXQ + window);
  }
  float m[4], l[4], o[4][4];
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    m[u] = -INFINITY;
    l[u] = 0.f;
#pragma unroll
    for (int t = 0; t < 4; ++t) o[u][t] = 0.f;
  }
  for (int j0 = lo; j0 < hi; j0 += kXK) {
    const int nk = min(kXK, hi - j0);
    __syncthreads();
    for (int i = threadIdx.x; i < nk * D; i += blockDim.x) {
      const int r = i / D, c = i % D;
      const int64_t off = kbase + (int64_t)(j0 + r) * kn + c;
      ks[r * DS + c] = to_f32(k[off]);
      vs[r * DS + c] = to_f32(v[off]);
    }
    __syncthreads();
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int qr = warp * 4 + u, qi = q0 + qr;
      if (qi >= Nq) continue;
      const float* qv = qs + qr * D;
      float sc[2];
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        const int jj = lane + 32 * t, j = j0 + jj;
        bool ok = jj < nk;
        if (ok && window >= 0) ok = (j - qi <= window) && (qi - j <= window);
        float acc = -INFINITY;
        if (ok) {
          const float* kr = ks + jj * DS;
          acc = 0.f;
          for (int c = 0; c < D; ++c) acc = fmaf(qv[c], kr[c], acc);
          acc *= scale;
        }
        sc[t] = acc;
      }
      const float mc = warp_max(fmaxf(sc[0], sc[1]));
      if (mc == -INFINITY) continue;
      const float mn = fmaxf(m[u], mc);
      const float corr = (m[u] == -INFINITY) ? 0.f : expf(m[u] - mn);
      const float p0 = (sc[0] == -INFINITY) ? 0.f : expf(sc[0] - mn);
      const float p1 = (sc[1] == -INFINITY) ? 0.f : expf(sc[1] - mn);
      l[u] = l[u] * corr + warp_sum(p0 + p1);
#pragma unroll
      for (int t = 0; t < 4; ++t) o[u][t] *= corr;
      for (int jj = 0; jj < nk; ++jj) {
        const float pj = __shfl_sync(MN_FULL_MASK, jj < 32 ? p0 : p1, jj & 31);
        if (pj == 0.f) continue;
        const float* vr = vs + jj * DS;
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const int c = lane + 32 * t;
          if (c < D) o[u][t] = fmaf(pj, vr[c], o[u][t]);
        }
      }
      m[u] = mn;
    }
  }
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int qi = q0 + warp * 4 + u;
    if (qi >= Nq) continue;
    const float inv = 1.0f / l[u];
    const int64_t ooff = (((int64_t)b * Nq + qi) * H + h) * D;
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const int c = lane + 32 * t;
      if (c < D) store_any(out, out_dtype, ooff + c, o[u][t] * inv);
    }
  }
}

}  // namespace mn

using namespace mn;

extern "C" int mn_attention(int batch, int nq, int nk, int heads, int head_dim, int dtype, const void* q,
                            int64_t q_sb, int64_t q_sn, int64_t q_sh, const void* k, const void* v, int64_t kv_sb,
                            int64_t kv_sn, int64_t kv_sh, int window, float scale, void* out, int out_dtype,
                            int* status, void* stream) {
  if (batch < 0 || nq < 0 || nk <= 0 || heads <= 0 || head_dim <= 0 || head_dim > 128 || !out) return MN_ERR_ARG;
  if ((int64_t)batch * nq == 0) return MN_OK;
  if (!q || !k || !v || dtype < 0 || dtype > 2 || out_dtype < 0 || out_dtype > 2) return MN_ERR_ARG;
  cudaGetLastError();
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  bool cls_unused = false;
  if (attention_tc(dtype, q, q_sb, q_sn, q_sh, k, v, kv_sb, kv_sn, kv_sh, batch, nq, nk, heads, head_dim, window,
                   scale, nullptr, 0, out, out_dtype, status, st, false, &cls_unused))
    return cudaGetLastError() == cudaSuccess ? MN_OK : MN_ERR_LAUNCH;
  const size_t smem = ((size_t)kXQ * head_dim + 2 * (size_t)kXK * (head_dim + 1)) * sizeof(float);
  const dim3 grid((nq + kXQ - 1) / kXQ, heads, batch);
  auto run = [&](auto tag) {
    using ET = decltype(tag);
    cudaFuncSetAttribute(attn_chunked_kernel<ET>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    attn_chunked_kernel<ET><<<grid, 256, smem, st>>>(static_cast<const ET*>(q), q_sb, q_sn, q_sh,
                                                     static_cast<const ET*>(k), static_cast<const ET*>(v), kv_sb,
                                                     kv_sn, kv_sh, nq, nk, heads, head_dim, window, scale, out,
                                                     out_dtype);
  };
  if (dtype == MN_F32) run(float{});
  else if (dtype == MN_F16) run(__half{});
  else run(__nv_bfloat16{});
  return cudaGetLastError() == cudaSuccess ? MN_OK : MN_ERR_LAUNCH;
}

extern "C" int mn_local_attention(int batch, int tokens, int heads, int head_dim, int dtype, const void* q,
                                  const void* k, const void* v, int64_t s_b, int64_t s_n, int64_t s_h,
                                  const void* bias, int bias_dtype, int window, int cls_global, float scale,
                                  void* out, int out_dtype, int* status, void* stream) {
  if (batch < 0 || tokens < 0 || heads <= 0 || head_dim <= 0 || head_dim > 128 || !out) return MN_ERR_ARG;
  if ((int64_t)batch * tokens == 0) return MN_OK;
  if (!q || !k || !v) return MN_ERR_ARG;
  if (dtype < 0 || dtype > 2 || out_dtype < 0 || out_dtype > 2 || (bias && (bias_dtype < 0 || bias_dtype > 2)))
    return MN_ERR_ARG;
  const int W = window < 0 ? tokens : window;
  const int nk = std::min(tokens, kLocalQT + 2 * W);
  const size_t smem = ((size_t)2 * nk * (head_dim + 1) + nk + 8 * head_dim) * sizeof(float);
  const bool tc_shape = head_dim == 64 && (dtype == MN_F16 || dtype == MN_BF16);
  if (smem > 200 * 1024 && !tc_shape) return MN_ERR_UNSUPPORTED;
  const bool cls_row = cls_global && window >= 0 && tokens > 1;
  // p[tokens], q[D] and the partial sums: at most 256 threads x 8 channels
  const size_t smem_cls = ((size_t)tokens + head_dim + 256 * 8) * sizeof(float);
  if (cls_row && (smem_cls > 200 * 1024 || head_dim > 256)) return MN_ERR_UNSUPPORTED;
  cudaGetLastError();
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const dim3 grid((tokens + kLocalQT - 1) / kLocalQT, heads, batch);
  bool cls_done = false;  // the tensor-core kernel computed the CLS row itself
  const bool tensor_core = attention_tc(dtype, q, s_b, s_n, s_h, k, v, s_b, s_n, s_h, batch, tokens, tokens, heads,
                                        head_dim, window, scale, bias, bias_dtype, out, out_dtype, status, st,
                                        cls_row, &cls_done);
  auto run = [&](auto tag) {
    using ET = decltype(tag);
    if (!tensor_core) {
      cudaFuncSetAttribute(local_attn_kernel<ET>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      local_attn_kernel<ET><<<grid, 256, smem, st>>>(static_cast<const ET*>(q), static_cast<const ET*>(k),
                                                     static_cast<const ET*>(v), s_b, s_n, s_h, tokens, heads,
                                                     head_dim, bias, bias_dtype, window, scale, out, out_dtype,
                                                     cls_row ? 1 : 0);
    }
    if (cls_row && !cls_done) {
      cudaFuncSetAttribute(cls_row_kernel<ET>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_cls);
      cls_row_kernel<ET><<<dim3(heads, batch), 256, smem_cls, st>>>(
          static_cast<const ET*>(q), static_cast<const ET*>(k), static_cast<const ET*>(v), s_b, s_n, s_h, tokens,
          heads, head_dim, bias, bias_dtype, scale, out, out_dtype);
    }
  };
  if (dtype == MN_F32) run(float{});
  else if (dtype == MN_F16) run(__half{});
  else run(__nv_bfloat16{});
  return cudaGetLastError() == cudaSuccess ? MN_OK : MN_ERR_LAUNCH;
}
