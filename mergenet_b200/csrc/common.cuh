// Shared device helpers for the MergeNet B200 kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <map>
#include <mutex>
#include <utility>

#include "../../include/mergenet_b200.h"

#define MN_FULL_MASK 0xffffffffu

// Packed fp32x2 arithmetic (sm_100): two independent round-to-nearest
// operations per instruction, bitwise equal to the scalar forms.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;"
      : "=l"(d)
      : "l"(*reinterpret_cast<const uint64_t*>(&a)), "l"(*reinterpret_cast<const uint64_t*>(&b)),
        "l"(*reinterpret_cast<const uint64_t*>(&c)));
  return *reinterpret_cast<const float2*>(&d);
}
__device__ __forceinline__ float2 fmul2(float2 a, float2 b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;"
      : "=l"(d)
      : "l"(*reinterpret_cast<const uint64_t*>(&a)), "l"(*reinterpret_cast<const uint64_t*>(&b)));
  return *reinterpret_cast<const float2*>(&d);
}
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;"
      : "=l"(d)
      : "l"(*reinterpret_cast<const uint64_t*>(&a)), "l"(*reinterpret_cast<const uint64_t*>(&b)));
  return *reinterpret_cast<const float2*>(&d);
}

namespace mn {

// ------------------------------------------------- dynamic shared memory
// Make sure `func` may launch with `bytes` of dynamic shared memory on the
// current device.  cudaFuncAttributeMaxDynamicSharedMemorySize is a
// process-wide setting per (device, kernel): if two host threads each set it
// to their own size before launching, one can lower the limit between the
// other's set and its launch.  Here the limit is only ever raised, under one
// lock, and the largest value set so far is remembered, so a launch never
// finds a limit below what it asked for.  Returns false if the driver
// refuses the size (nothing should be launched then).
inline bool ensure_dynamic_smem(const void* func, size_t bytes) {
  static std::mutex mu;
  static std::map<std::pair<int, const void*>, size_t> set_so_far;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  std::lock_guard<std::mutex> lock(mu);
  size_t& cur = set_so_far[{dev, func}];
  if (bytes <= cur) return true;
  if (cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) != cudaSuccess) {
    cudaGetLastError();  // the refusal is reported by the return value, not left sticky
    return false;
  }
  cur = bytes;
  return true;
}
template <typename F>
inline bool ensure_smem(F* func, size_t bytes) {
  return ensure_dynamic_smem(reinterpret_cast<const void*>(func), bytes);
}

// ---------------------------------------------------------------- dtype I/O
template <int DT> struct Elem;
template <> struct Elem<MN_F32> { using T = float; };
template <> struct Elem<MN_F16> { using T = __half; };
template <> struct Elem<MN_BF16> { using T = __nv_bfloat16; };

__device__ __forceinline__ float to_f32(float v) { return v; }
__device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }
__device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

// Load element i of a buffer whose dtype is only known at run time.
__device__ __forceinline__ float load_any(const void* p, int dtype, int64_t i) {
  if (dtype == MN_F32) return static_cast<const float*>(p)[i];
  if (dtype == MN_F16) return __half2float(static_cast<const __half*>(p)[i]);
  return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
}
__device__ __forceinline__ void store_any(void* p, int dtype, int64_t i, float v) {
  if (dtype == MN_F32) static_cast<float*>(p)[i] = v;
  else if (dtype == MN_F16) static_cast<__half*>(p)[i] = __float2half_rn(v);
  else static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
}

// ---------------------------------------------------------- warp reductions
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(MN_FULL_MASK, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(MN_FULL_MASK, v, o));
  return v;
}
__device__ __forceinline__ float warp_min(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fminf(v, __shfl_xor_sync(MN_FULL_MASK, v, o));
  return v;
}
__device__ __forceinline__ int warp_min_int(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = min(v, __shfl_xor_sync(MN_FULL_MASK, v, o));
  return v;
}

// Block-wide min/max of one float per thread (blockDim.x multiple of 32,
// <= 1024).  scratch: >= 64 floats of shared memory.  Result in every thread.
__device__ __forceinline__ void block_minmax(float& vmin, float& vmax, float* scratch) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  vmin = warp_min(vmin);
  vmax = warp_max(vmax);
  __syncthreads();
  if (lane == 0) { scratch[warp] = vmin; scratch[32 + warp] = vmax; }
  __syncthreads();
  float a = (lane < nw) ? scratch[lane] : INFINITY;
  float b = (lane < nw) ? scratch[32 + lane] : -INFINITY;
  vmin = warp_min(a);
  vmax = warp_max(b);
  __syncthreads();
}

// Block-wide sum of one float per thread (fixed order: warp trees, then the
// warps' sums in warp order).  scratch: >= 32 floats.  Result in every thread.
__device__ __forceinline__ float block_sum(float v, float* scratch) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  v = warp_sum((lane < nw) ? scratch[lane] : 0.f);
  __syncthreads();
  return v;
}

__device__ __forceinline__ int block_min_int(int v, int* scratch) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_min_int(v);
  __syncthreads();
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  int a = (lane < nw) ? scratch[lane] : 0x7fffffff;
  v = warp_min_int(a);
  __syncthreads();
  return v;
}

// Inclusive block scan of doubles; each thread owns `per` consecutive
// elements of buf[0 .. blockDim.x*per).  scratch: >= 32 doubles.
__device__ __forceinline__ void block_scan_inclusive(double* buf, int per, double* scratch) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  double* mine = buf + threadIdx.x * per;
  double run = 0.0;
  for (int i = 0; i < per; ++i) { run += mine[i]; mine[i] = run; }
  double incl = run;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    double t = __shfl_up_sync(MN_FULL_MASK, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) scratch[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    double w = (lane < nw) ? scratch[lane] : 0.0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      double t = __shfl_up_sync(MN_FULL_MASK, w, o);
      if (lane >= o) w += t;
    }
    if (lane < nw) scratch[lane] = w;
  }
  __syncthreads();
  double offset = (incl - run) + (warp > 0 ? scratch[warp - 1] : 0.0);
  for (int i = 0; i < per; ++i) mine[i] += offset;
  __syncthreads();
}

// Ascending bitonic sort of n (power of two) floats in shared memory.  With
// one element per thread (n == blockDim.x) each thread keeps its element in a
// register: exchanges within a warp are shuffles, wider ones go through s
// (two barriers each) -- 10 barrier pairs instead of 45 barriers at n = 512.
__device__ __forceinline__ void bitonic_sort_f32(float* s, int n) {
  if (n == (int)blockDim.x && n >= 32) {
    const int i = threadIdx.x;
    float key = s[i];
    for (int k = 2; k <= n; k <<= 1) {
      for (int j = k >> 1; j > 0; j >>= 1) {
        float other;
        if (j >= 32) {
          s[i] = key;
          __syncthreads();
          other = s[i ^ j];
          __syncthreads();
        } else {
          other = __shfl_xor_sync(MN_FULL_MASK, key, j);
        }
        const bool up = (i & k) == 0, lower = (i & j) == 0;
        const float lo = (key > other) ? other : key, hi = (key > other) ? key : other;
        key = (lower == up) ? lo : hi;
      }
    }
    s[i] = key;
    __syncthreads();
    return;
  }
  for (int k = 2; k <= n; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < n; i += blockDim.x) {
        int ixj = i ^ j;
        if (ixj > i) {
          float a = s[i], b = s[ixj];
          bool up = (i & k) == 0;
          if ((a > b) == up) { s[i] = b; s[ixj] = a; }
        }
      }
      __syncthreads();
    }
  }
}

// Ascending bitonic sort of n (power of two) 64-bit keys in shared memory.
__device__ __forceinline__ void bitonic_sort_u64(unsigned long long* s, int n) {
  for (int k = 2; k <= n; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < n; i += blockDim.x) {
        int ixj = i ^ j;
        if (ixj > i) {
          unsigned long long a = s[i], b = s[ixj];
          bool up = (i & k) == 0;
          if ((a > b) == up) { s[i] = b; s[ixj] = a; }
        }
      }
      __syncthreads();
    }
  }
}

// Bitonic sort of n keys (n a power of two, n <= R * blockDim.x,
// blockDim.x a power of two >= 32) held in registers: thread i holds the
// keys at positions i + r * blockDim.x (r = 0 .. R-1) in kv[r] and receives
// those positions of the ascending order.  Positions at or past n must hold
// keys that sort last (~0 for integers, +inf for floats).  Partners R * blockDim.x / 2 .. blockDim.x apart
// are the thread's own registers, partners under 32 apart are reached by warp
// shuffles, and the steps in between exchange through `xbuf` (2 * R *
// blockDim.x keys of shared memory, double-buffered: one barrier per step).
// Every thread of the block must call it with the same n.
template <int R, typename K>
__device__ __forceinline__ void bitonic_sort_regs(K (&kv)[R], K* xbuf, int n) {
  const int bd = blockDim.x;
  const int i = threadIdx.x;
  int parity = 0;
  auto pick = [](K key, K other, int idx, int k, int j) {
    const bool up = (idx & k) == 0, lower = (idx & j) == 0;
    const K lo = key > other ? other : key, hi = key > other ? key : other;
    return (lower == up) ? lo : hi;
  };
  for (int k = 2; k <= n; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      if (j >= bd) {  // partner r ^ (j / bd) of the thread's own keys
#pragma unroll
        for (int t = 1; t < R; t <<= 1) {
          if (j == t * bd) {
#pragma unroll
            for (int r = 0; r < R; ++r) {
              if ((r & t) == 0) {
                const bool up = ((i + r * bd) & k) == 0;
                const K a = kv[r], b = kv[r | t];
                const bool sw = up ? (a > b) : (a < b);
                kv[r] = sw ? b : a;
                kv[r | t] = sw ? a : b;
              }
            }
          }
        }
      } else if (j >= 32) {
        K* buf = xbuf + parity * R * bd;
#pragma unroll
        for (int r = 0; r < R; ++r) buf[i + r * bd] = kv[r];
        __syncthreads();
#pragma unroll
        for (int r = 0; r < R; ++r) kv[r] = pick(kv[r], buf[(i + r * bd) ^ j], i + r * bd, k, j);
        parity ^= 1;
      } else {
#pragma unroll
        for (int r = 0; r < R; ++r)
          kv[r] = pick(kv[r], __shfl_xor_sync(MN_FULL_MASK, kv[r], j), i + r * bd, k, j);
      }
    }
  }
}

__host__ __device__ inline int next_pow2(int v) {
  int p = 1;
  while (p < v) p <<= 1;
  return p;
}

}  // namespace mn
