// Fused residual add + LayerNorm + fp16 cast for the fp32 residual streams of
// the local and latent blocks.  Under fp16 autocast the reference computes
// x = x + f(...) in fp32, LayerNorm in fp32 and casts the result to fp16 for
// the next Linear (timm Block / LocalBlock forward,
// opentome/timm/bias_local_attn.py:867-868); here one pass reads x (and the
// fp16 branch output) once and writes the fp32 sum and the fp16 LayerNorm.
#include "common.cuh"

namespace mn {

// Four floats <-> four 16-bit values (fp16 or bf16) as one 8-byte word.
template <typename HT>
__device__ __forceinline__ uint2 pack4(float a, float b, float c, float d) {
  HT h[4] = {from_f32<HT>(a), from_f32<HT>(b), from_f32<HT>(c), from_f32<HT>(d)};
  return *reinterpret_cast<const uint2*>(h);
}
template <typename HT>
__device__ __forceinline__ void unpack4(uint2 u, float* f) {
  const HT* h = reinterpret_cast<const HT*>(&u);
#pragma unroll
  for (int j = 0; j < 4; ++j) f[j] = to_f32(h[j]);
}

// 16-bit (HT) LayerNorm of one row held by a warp (four floats per lane-step).
template <int C, typename HT>
__device__ __forceinline__ void layernorm_row_store(const float (&v)[C / 128][4], const float* __restrict__ gamma,
                                                    const float* __restrict__ beta, float eps, HT* hrow,
                                                    int lane) {
  constexpr int V = C / 128;
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < V; ++i) s += (v[i][0] + v[i][1]) + (v[i][2] + v[i][3]);
  const float mean = warp_sum(s) * (1.0f / C);
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < V; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float d = v[i][j] - mean;
      q = fmaf(d, d, q);
    }
  const float rstd = rsqrtf(warp_sum(q) * (1.0f / C) + eps);
  const float4* g4 = reinterpret_cast<const float4*>(gamma);
  const float4* b4 = reinterpret_cast<const float4*>(beta);
  uint2* hl = reinterpret_cast<uint2*>(hrow);
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const float4 g = g4[lane + 32 * i], bb = b4[lane + 32 * i];
    const float o0 = (v[i][0] - mean) * rstd * g.x + bb.x, o1 = (v[i][1] - mean) * rstd * g.y + bb.y;
    const float o2 = (v[i][2] - mean) * rstd * g.z + bb.z, o3 = (v[i][3] - mean) * rstd * g.w + bb.w;
    hl[lane + 32 * i] = pack4<HT>(o0, o1, o2, o3);
  }
}

// One warp per row; C must be a multiple of 128 (four floats per lane-step).
template <int C, typename HT>
__global__ void __launch_bounds__(256) add_layernorm_kernel(const float* __restrict__ x, const HT* __restrict__ y,
                                                            const float* __restrict__ gamma,
                                                            const float* __restrict__ beta, float eps, int64_t rows,
                                                            float* __restrict__ x_out, HT* __restrict__ h_ln,
                                                            HT* __restrict__ h_raw) {
  constexpr int V = C / 128;  // float4 groups per lane
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float4* xr = reinterpret_cast<const float4*>(x + row * C);
  float v[V][4];
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const float4 a = xr[lane + 32 * i];
    v[i][0] = a.x; v[i][1] = a.y; v[i][2] = a.z; v[i][3] = a.w;
  }
  if (y) {
    const uint2* yr = reinterpret_cast<const uint2*>(y + row * C);
#pragma unroll
    for (int i = 0; i < V; ++i) {
      float f[4];
      unpack4<HT>(yr[lane + 32 * i], f);
      v[i][0] += f[0]; v[i][1] += f[1];
      v[i][2] += f[2]; v[i][3] += f[3];
    }
  }
  if (x_out) {
    float4* xo = reinterpret_cast<float4*>(x_out + row * C);
#pragma unroll
    for (int i = 0; i < V; ++i) xo[lane + 32 * i] = make_float4(v[i][0], v[i][1], v[i][2], v[i][3]);
  }
  if (h_raw) {
    uint2* hr = reinterpret_cast<uint2*>(h_raw + row * C);
#pragma unroll
    for (int i = 0; i < V; ++i) hr[lane + 32 * i] = pack4<HT>(v[i][0], v[i][1], v[i][2], v[i][3]);
  }
  if (h_ln) layernorm_row_store<C, HT>(v, gamma, beta, eps, h_ln + row * C, lane);
}

// LayerNorm(x + y) of one row per warp, written in fp32: the latent
// encoder's final norm, which autocast runs in fp32 (model.py:1195-1198).
template <int C, typename HT>
__global__ void __launch_bounds__(256) add_layernorm_f32_kernel(const float* __restrict__ x,
                                                                const HT* __restrict__ y,
                                                                const float* __restrict__ gamma,
                                                                const float* __restrict__ beta, float eps,
                                                                int64_t rows, float* __restrict__ out) {
  constexpr int V = C / 128;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float4* xr = reinterpret_cast<const float4*>(x + row * C);
  float v[V][4];
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const float4 a = xr[lane + 32 * i];
    v[i][0] = a.x; v[i][1] = a.y; v[i][2] = a.z; v[i][3] = a.w;
  }
  if (y) {
    const uint2* yr = reinterpret_cast<const uint2*>(y + row * C);
#pragma unroll
    for (int i = 0; i < V; ++i) {
      float f[4];
      unpack4<HT>(yr[lane + 32 * i], f);
      v[i][0] += f[0]; v[i][1] += f[1];
      v[i][2] += f[2]; v[i][3] += f[3];
    }
  }
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < V; ++i) s += (v[i][0] + v[i][1]) + (v[i][2] + v[i][3]);
  const float mean = warp_sum(s) * (1.0f / C);
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < V; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float d = v[i][j] - mean;
      q = fmaf(d, d, q);
    }
  const float rstd = rsqrtf(warp_sum(q) * (1.0f / C) + eps);
  const float4* g4 = reinterpret_cast<const float4*>(gamma);
  const float4* b4 = reinterpret_cast<const float4*>(beta);
  float4* o = reinterpret_cast<float4*>(out + row * C);
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const float4 g = g4[lane + 32 * i], bb = b4[lane + 32 * i];
    o[lane + 32 * i] = make_float4((v[i][0] - mean) * rstd * g.x + bb.x, (v[i][1] - mean) * rstd * g.y + bb.y,
                                   (v[i][2] - mean) * rstd * g.z + bb.z, (v[i][3] - mean) * rstd * g.w + bb.w);
  }
}

// fp32 LayerNorm of one row per warp, written as two fp16 planes for the
// split-precision GEMM: ys = LayerNorm(x) * scale (scale an exact power of
// two), hi = fp16(ys), lo = fp16(ys - hi), so hi + lo carries ys to 2^-22.
template <int C>
__global__ void __launch_bounds__(256) layernorm_split_kernel(const float* __restrict__ x,
                                                              const float* __restrict__ gamma,
                                                              const float* __restrict__ beta, float eps, float scale,
                                                              int64_t rows, __half* __restrict__ hi_out,
                                                              __half* __restrict__ lo_out) {
  constexpr int V = C / 128;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float4* xr = reinterpret_cast<const float4*>(x + row * C);
  float v[V][4];
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const float4 a = xr[lane + 32 * i];
    v[i][0] = a.x; v[i][1] = a.y; v[i][2] = a.z; v[i][3] = a.w;
  }
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < V; ++i) s += (v[i][0] + v[i][1]) + (v[i][2] + v[i][3]);
  const float mean = warp_sum(s) * (1.0f / C);
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < V; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float d = v[i][j] - mean;
      q = fmaf(d, d, q);
    }
  const float rstd = rsqrtf(warp_sum(q) * (1.0f / C) + eps);
  const float4* g4 = reinterpret_cast<const float4*>(gamma);
  const float4* b4 = reinterpret_cast<const float4*>(beta);
  uint2* hrow = reinterpret_cast<uint2*>(hi_out + row * C);
  uint2* lrow = reinterpret_cast<uint2*>(lo_out + row * C);
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const float4 g = g4[lane + 32 * i], bb = b4[lane + 32 * i];
    float o[4] = {(v[i][0] - mean) * rstd * g.x + bb.x, (v[i][1] - mean) * rstd * g.y + bb.y,
                  (v[i][2] - mean) * rstd * g.z + bb.z, (v[i][3] - mean) * rstd * g.w + bb.w};
    __half h[4], l[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float ys = o[j] * scale;
      h[j] = __float2half_rn(ys);
      l[j] = __float2half_rn(ys - __half2float(h[j]));
    }
    hrow[lane + 32 * i] = *reinterpret_cast<const uint2*>(h);
    lrow[lane + 32 * i] = *reinterpret_cast<const uint2*>(l);
  }
}

// The embedding step of the local ViT fused with the first block's LayerNorm
// (timm PatchEmbed + _pos_embed, then norm1): row t of image b is
// cls + pos[0] for t == 0 and float(emb[b, t - 1]) + pos[t] otherwise, with
// emb the fp16 patch-projection output.  Writes that fp32 row and its fp16
// LayerNorm.
template <int C, typename HT>
__global__ void __launch_bounds__(256) embed_layernorm_kernel(const HT* __restrict__ emb,
                                                              const float* __restrict__ pos,
                                                              const float* __restrict__ cls, int tokens,
                                                              const float* __restrict__ gamma,
                                                              const float* __restrict__ beta, float eps,
                                                              int64_t rows, float* __restrict__ x_out,
                                                              HT* __restrict__ h_ln) {
  constexpr int V = C / 128;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int t = (int)(row % tokens);
  const int64_t b = row / tokens;
  const float4* pr = reinterpret_cast<const float4*>(pos + (int64_t)t * C);
  float v[V][4];
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const float4 a = pr[lane + 32 * i];
    v[i][0] = a.x; v[i][1] = a.y; v[i][2] = a.z; v[i][3] = a.w;
  }
  if (t == 0) {
    const float4* cr = reinterpret_cast<const float4*>(cls);
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const float4 a = cr[lane + 32 * i];
      v[i][0] = a.x + v[i][0]; v[i][1] = a.y + v[i][1]; v[i][2] = a.z + v[i][2]; v[i][3] = a.w + v[i][3];
    }
  } else {
    const uint2* er = reinterpret_cast<const uint2*>(emb + (b * (tokens - 1) + (t - 1)) * C);
#pragma unroll
    for (int i = 0; i < V; ++i) {
      float f[4];
      unpack4<HT>(er[lane + 32 * i], f);
      v[i][0] = f[0] + v[i][0]; v[i][1] = f[1] + v[i][1];
      v[i][2] = f[2] + v[i][2]; v[i][3] = f[3] + v[i][3];
    }
  }
  float4* xo = reinterpret_cast<float4*>(x_out + row * C);
#pragma unroll
  for (int i = 0; i < V; ++i) xo[lane + 32 * i] = make_float4(v[i][0], v[i][1], v[i][2], v[i][3]);
  layernorm_row_store<C, HT>(v, gamma, beta, eps, h_ln + row * C, lane);
}

}  // namespace mn

using namespace mn;

extern "C" int mn_add_layernorm(int64_t rows, int channels, const float* x, const void* y, const float* gamma,
                                const float* beta, float eps, float* x_out, void* h_ln, void* h_raw, int half_dtype,
                                void* stream) {
  if (rows < 0 || channels <= 0) return MN_ERR_ARG;
  if (rows == 0) return MN_OK;
  if (!x || (h_ln && (!gamma || !beta))) return MN_ERR_ARG;
  if (half_dtype != MN_F16 && half_dtype != MN_BF16) return MN_ERR_ARG;
  cudaGetLastError();
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned grid = (unsigned)((rows + 7) / 8);
  auto run = [&](auto tag) {
    using HT = decltype(tag);
    const HT* yh = static_cast<const HT*>(y);
    HT* hl = static_cast<HT*>(h_ln);
    HT* hr = static_cast<HT*>(h_raw);
    switch (channels) {
      case 384: add_layernorm_kernel<384, HT><<<grid, 256, 0, st>>>(x, yh, gamma, beta, eps, rows, x_out, hl, hr); return true;
      case 256: add_layernorm_kernel<256, HT><<<grid, 256, 0, st>>>(x, yh, gamma, beta, eps, rows, x_out, hl, hr); return true;
      case 512: add_layernorm_kernel<512, HT><<<grid, 256, 0, st>>>(x, yh, gamma, beta, eps, rows, x_out, hl, hr); return true;
      case 768: add_layernorm_kernel<768, HT><<<grid, 256, 0, st>>>(x, yh, gamma, beta, eps, rows, x_out, hl, hr); return true;
      default: return false;
    }
  };
  const bool ok = half_dtype == MN_F16 ? run(__half{}) : run(__nv_bfloat16{});
  if (!ok) return MN_ERR_UNSUPPORTED;
  return cudaGetLastError() == cudaSuccess ? MN_OK : MN_ERR_LAUNCH;
}

extern "C" int mn_embed_layernorm(int batch, int tokens, int channels, const void* emb, const float* pos,
                                  const float* cls, const float* gamma, const float* beta, float eps, float* x_out,
                                  void* h_ln, int half_dtype, void* stream) {
  if (batch < 0 || tokens < 1 || channels <= 0) return MN_ERR_ARG;
  if (batch == 0) return MN_OK;
  if ((tokens > 1 && !emb) || !pos || !cls || !gamma || !beta || !x_out || !h_ln) return MN_ERR_ARG;
  if (half_dtype != MN_F16 && half_dtype != MN_BF16) return MN_ERR_ARG;
  cudaGetLastError();
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t rows = (int64_t)batch * tokens;
  const unsigned grid = (unsigned)((rows + 7) / 8);
  auto run = [&](auto tag) {
    using HT = decltype(tag);
    const HT* e = static_cast<const HT*>(emb);
    HT* hl = static_cast<HT*>(h_ln);
    switch (channels) {
      case 384: embed_layernorm_kernel<384, HT><<<grid, 256, 0, st>>>(e, pos, cls, tokens, gamma, beta, eps, rows, x_out, hl); return true;
      case 256: embed_layernorm_kernel<256, HT><<<grid, 256, 0, st>>>(e, pos, cls, tokens, gamma, beta, eps, rows, x_out, hl); return true;
      case 512: embed_layernorm_kernel<512, HT><<<grid, 256, 0, st>>>(e, pos, cls, tokens, gamma, beta, eps, rows, x_out, hl); return true;
      case 768: embed_layernorm_kernel<768, HT><<<grid, 256, 0, st>>>(e, pos, cls, tokens, gamma, beta, eps, rows, x_out, hl); return true;
      default: return false;
    }
  };
  const bool ok = half_dtype == MN_F16 ? run(__half{}) : run(__nv_bfloat16{});
  if (!ok) return MN_ERR_UNSUPPORTED;
  return cudaGetLastError() == cudaSuccess ? MN_OK : MN_ERR_LAUNCH;
}

// Patch unfold of the patch-embedding convolution (timm PatchEmbed, a
// stride-p p x p conv, computed as one GEMM over unfolded patches): images
// fp32 [B, C, H, W] -> patches fp16 [B, H/p, W/p, C, p, p] (row = one patch,
// C*p*p contiguous values, the conv weight's [C, p, p] order).  One thread
// per 8-value run of a patch row: a 32-byte read of the image row and a
// 16-byte write; consecutive threads write consecutive output bytes.
__global__ void __launch_bounds__(256) patch_unfold_kernel(const float* __restrict__ img, int C, int Hh, int Ww,
                                                           int p, int64_t total, __half* __restrict__ out) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= total) return;
  const int runs = C * p * p / 8;  // 8-value runs per patch
  const int64_t patch = t / runs;
  const int r = (int)(t % runs);
  const int gw = Ww / p, gh = Hh / p;
  const int gx = (int)(patch % gw);
  const int64_t rest = patch / gw;
  const int gy = (int)(rest % gh);
  const int64_t b = rest / gh;
  const int per_c = p * p / 8;
  const int c = r / per_c, rr = r % per_c;
  const int py = rr / (p / 8), px0 = (rr % (p / 8)) * 8;
  const float4* src = reinterpret_cast<const float4*>(img + (((b * C + c) * Hh + gy * p + py) * (int64_t)Ww + gx * p + px0));
  const float4 a = __ldg(src), d = __ldg(src + 1);
  __half2 h0 = __floats2half2_rn(a.x, a.y), h1 = __floats2half2_rn(a.z, a.w);
  __half2 h2 = __floats2half2_rn(d.x, d.y), h3 = __floats2half2_rn(d.z, d.w);
  uint4 u;
  u.x = *reinterpret_cast<uint32_t*>(&h0);
  u.y = *reinterpret_cast<uint32_t*>(&h1);
  u.z = *reinterpret_cast<uint32_t*>(&h2);
  u.w = *reinterpret_cast<uint32_t*>(&h3);
  reinterpret_cast<uint4*>(out)[t] = u;
}

extern "C" int mn_patch_unfold(int batch, int channels, int height, int width, int patch, const float* images,
                               void* out, void* stream) {
  if (batch < 0 || channels <= 0 || patch <= 0 || height <= 0 || width <= 0) return MN_ERR_ARG;
  if (height % patch != 0 || width % patch != 0) return MN_ERR_ARG;
  if (batch == 0) return MN_OK;
  if (!images || !out) return MN_ERR_ARG;
  // 16-byte runs: p a multiple of 8, aligned rows and buffers
  if (patch % 8 != 0 || width % 4 != 0 || reinterpret_cast<uintptr_t>(images) % 16 != 0 ||
      reinterpret_cast<uintptr_t>(out) % 16 != 0)
    return MN_ERR_UNSUPPORTED;
  cudaGetLastError();
  const int64_t total = (int64_t)batch * (height / patch) * (width / patch) * channels * patch * patch / 8;
  patch_unfold_kernel<<<(unsigned)((total + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      images, channels, height, width, patch, total, static_cast<__half*>(out));
  return cudaGetLastError() == cudaSuccess ? MN_OK : MN_ERR_LAUNCH;
}

extern "C" int mn_layernorm_split(int64_t rows, int channels, const float* x, const float* gamma, const float* beta,
                                  float eps, float scale, void* hi, void* lo, void* stream) {
  if (rows < 0 || channels <= 0) return MN_ERR_ARG;
  if (rows == 0) return MN_OK;
  if (!x || !gamma || !beta || !hi || !lo) return MN_ERR_ARG;
  cudaGetLastError();
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned grid = (unsigned)((rows + 7) / 8);
  __half* h = static_cast<__half*>(hi);
  __half* l = static_cast<__half*>(lo);
  switch (channels) {
    case 384: layernorm_split_kernel<384><<<grid, 256, 0, st>>>(x, gamma, beta, eps, scale, rows, h, l); break;
    case 256: layernorm_split_kernel<256><<<grid, 256, 0, st>>>(x, gamma, beta, eps, scale, rows, h, l); break;
    case 512: layernorm_split_kernel<512><<<grid, 256, 0, st>>>(x, gamma, beta, eps, scale, rows, h, l); break;
    case 768: layernorm_split_kernel<768><<<grid, 256, 0, st>>>(x, gamma, beta, eps, scale, rows, h, l); break;
    default: return MN_ERR_UNSUPPORTED;
  }
  return cudaGetLastError() == cudaSuccess ? MN_OK : MN_ERR_LAUNCH;
}

extern "C" int mn_add_layernorm_f32(int64_t rows, int channels, const float* x, const void* y, const float* gamma,
                                    const float* beta, float eps, float* out, int half_dtype, void* stream) {
  if (rows < 0 || !x || !gamma || !beta || !out) return MN_ERR_ARG;
  if (rows == 0) return MN_OK;
  if (half_dtype != MN_F16 && half_dtype != MN_BF16) return MN_ERR_ARG;
  cudaGetLastError();
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned grid = (unsigned)((rows + 7) / 8);
  auto run = [&](auto tag) -> bool {
    using HT = decltype(tag);
    const HT* yh = static_cast<const HT*>(y);
    switch (channels) {
      case 384: add_layernorm_f32_kernel<384, HT><<<grid, 256, 0, st>>>(x, yh, gamma, beta, eps, rows, out); return true;
      case 256: add_layernorm_f32_kernel<256, HT><<<grid, 256, 0, st>>>(x, yh, gamma, beta, eps, rows, out); return true;
      case 512: add_layernorm_f32_kernel<512, HT><<<grid, 256, 0, st>>>(x, yh, gamma, beta, eps, rows, out); return true;
      case 768: add_layernorm_f32_kernel<768, HT><<<grid, 256, 0, st>>>(x, yh, gamma, beta, eps, rows, out); return true;
      default: return false;
    }
  };
  const bool ok = half_dtype == MN_F16 ? run(__half{}) : run(__nv_bfloat16{});
  if (!ok) return MN_ERR_UNSUPPORTED;
  return cudaGetLastError() == cudaSuccess ? MN_OK : MN_ERR_LAUNCH;
}
