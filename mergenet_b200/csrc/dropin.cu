// Function-level drop-ins for the reference's routing primitives, for
// arbitrary donor/receiver partitions (training grouping, seeded grouping,
// odd grids): the fused path in route.cu covers only the canonical eval
// grouping.
#include <algorithm>
#include <map>
#include <mutex>

#include "common.cuh"
#include "thretopk.cuh"

namespace mn {

// --------------------------------------------------------------------------
// sparse_spatial_score (dtem.py:361-433 / :554-594): per (batch, donor) one
// warp.  Lanes resolve the static neighbour -> receiver slot by a left
// binary search in the sorted receiver list (static-invalid slots map to 0),
// then the warp computes each valid slot's fp32 dot product.
// --------------------------------------------------------------------------
// QUAD: rows of whole 64-byte groups, 16-byte aligned: four lanes share a
// slot's dot product (lane q takes the row's 16-byte vectors q, q + 4, ...)
// and a warp scores eight slots at a time.
template <typename ET, bool QUAD>
__global__ void __launch_bounds__(256) sparse_score_kernel(
    const ET* __restrict__ a, const ET* __restrict__ b, const int64_t* __restrict__ nbr,
    const uint8_t* __restrict__ nbr_valid, const int64_t* __restrict__ donor_patch,
    const int64_t* __restrict__ recv_patch, int B, int Na, int Nb, int P, int K, int C,
    ET* __restrict__ scores, int64_t* __restrict__ ridx_out, uint8_t* __restrict__ rvalid_out) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= (int64_t)B * Na) return;
  const int bb = (int)(row / Na);
  const int64_t pd = donor_patch[row];
  const int64_t* rp = recv_patch + (int64_t)bb * Nb;
  const ET* arow = a + row * C;
  for (int k0 = 0; k0 < K; k0 += 32) {
    const int k = k0 + lane;
    int64_t slot = 0;
    bool ok = false;
    if (k < K && pd >= 0 && pd < P) {
      const int64_t t = pd * K + k;
      if (nbr_valid[t]) {
        const int64_t n = nbr[t];
        int lo = 0, hi = Nb;
        while (lo < hi) {
          int mid = (lo + hi) >> 1;
          if (rp[mid] < n) lo = mid + 1; else hi = mid;
        }
        slot = lo < Nb ? lo : Nb - 1;
        ok = lo < Nb && rp[slot] == n;
      }
    }
    const int kmax = min(32, K - k0);
    if constexpr (QUAD) {
      constexpr int E = 16 / sizeof(ET);  // elements per 16-byte vector
      const int vpr = C / E;              // vectors per row, a multiple of 4
      const int q = lane & 3;
      for (int g = 0; g < kmax; g += 8) {
        const int j = g + (lane >> 2);
        const int jj = min(j, kmax - 1);
        const int64_t s = __shfl_sync(MN_FULL_MASK, slot, jj);
        const bool v = __shfl_sync(MN_FULL_MASK, ok, jj) && j < kmax;
        float acc = 0.f;
        if (v) {
          const uint4* av = reinterpret_cast<const uint4*>(arow);
          const uint4* bv = reinterpret_cast<const uint4*>(b + ((int64_t)bb * Nb + s) * C);
          for (int t = q; t < vpr; t += 4) {
            const uint4 ua = av[t], ub = bv[t];
            const ET* ea = reinterpret_cast<const ET*>(&ua);
            const ET* eb = reinterpret_cast<const ET*>(&ub);
#pragma unroll
            for (int e = 0; e < E; ++e) acc = fmaf(to_f32(ea[e]), to_f32(eb[e]), acc);
          }
        }
        acc += __shfl_xor_sync(MN_FULL_MASK, acc, 1);
        acc += __shfl_xor_sync(MN_FULL_MASK, acc, 2);
        if (q == 0 && j < kmax) {
          const int64_t o = row * K + k0 + j;
          scores[o] = from_f32<ET>(acc);
          ridx_out[o] = s;
          rvalid_out[o] = v ? 1 : 0;
        }
      }
    } else {
      for (int j = 0; j < kmax; ++j) {
        const int64_t s = __shfl_sync(MN_FULL_MASK, slot, j);
        const bool v = __shfl_sync(MN_FULL_MASK, ok, j);
        float acc = 0.f;
        if (v) {
          const ET* brow = b + ((int64_t)bb * Nb + s) * C;
          for (int c = lane; c < C; c += 32) acc = fmaf(to_f32(arow[c]), to_f32(brow[c]), acc);
          acc = warp_sum(acc);
        }
        if (lane == 0) {
          const int64_t o = row * K + k0 + j;
          scores[o] = from_f32<ET>(acc);
          ridx_out[o] = s;
          rvalid_out[o] = v ? 1 : 0;
        }
      }
    }
  }
}

// sparse_neighbor_dot (dtem.py:286-315): same dot with precomputed slots.
// QUAD as in sparse_score_kernel: four lanes per slot, eight slots a pass.
template <typename ET, bool QUAD>
__global__ void __launch_bounds__(256) neighbor_dot_kernel(
    const ET* __restrict__ a, const ET* __restrict__ b, const int64_t* __restrict__ ridx,
    const uint8_t* __restrict__ rvalid, int B, int Na, int Nb, int K, int C, ET* __restrict__ scores) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= (int64_t)B * Na) return;
  const int bb = (int)(row / Na);
  const ET* arow = a + row * C;
  if constexpr (QUAD) {
    constexpr int E = 16 / sizeof(ET);
    const int vpr = C / E;
    const int q = lane & 3;
    for (int g = 0; g < K; g += 8) {
      const int k = g + (lane >> 2);
      const int64_t o = row * K + min(k, K - 1);
      const int64_t s = ridx[o];
      const bool v = k < K && rvalid[o] != 0 && s >= 0 && s < Nb;
      float acc = 0.f;
      if (v) {
        const uint4* av = reinterpret_cast<const uint4*>(arow);
        const uint4* bv = reinterpret_cast<const uint4*>(b + ((int64_t)bb * Nb + s) * C);
        for (int t = q; t < vpr; t += 4) {
          const uint4 ua = av[t], ub = bv[t];
          const ET* ea = reinterpret_cast<const ET*>(&ua);
          const ET* eb = reinterpret_cast<const ET*>(&ub);
#pragma unroll
          for (int e = 0; e < E; ++e) acc = fmaf(to_f32(ea[e]), to_f32(eb[e]), acc);
        }
      }
      acc += __shfl_xor_sync(MN_FULL_MASK, acc, 1);
      acc += __shfl_xor_sync(MN_FULL_MASK, acc, 2);
      if (q == 0 && k < K) scores[row * K + k] = from_f32<ET>(acc);
    }
  } else {
    for (int k = 0; k < K; ++k) {
      const int64_t o = row * K + k;
      const bool v = rvalid[o] != 0;
      const int64_t s = ridx[o];
      float acc = 0.f;
      if (v && s >= 0 && s < Nb) {
        const ET* brow = b + ((int64_t)bb * Nb + s) * C;
        for (int c = lane; c < C; c += 32) acc = fmaf(to_f32(arow[c]), to_f32(brow[c]), acc);
        acc = warp_sum(acc);
      }
      if (lane == 0) scores[o] = from_f32<ET>(acc);
    }
  }
}

// --------------------------------------------------------------------------
// sparse_weighted_transport without atomics (dtem.py:436-468, CPU order
// :911-926): each CTA (batch, channel chunk) builds receiver-centric edge
// lists in shared memory with a stable counting sort (ascending edge id, the
// reference's sequential scatter order), then gathers.
// --------------------------------------------------------------------------
template <typename ET>
__global__ void __launch_bounds__(512) transport_kernel(
    const ET* __restrict__ w, const ET* __restrict__ v, const int64_t* __restrict__ ridx,
    const uint8_t* __restrict__ rvalid, int Na, int Nb, int K, int C, int CC, int sort_warps,
    ET* __restrict__ out, int* status) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  int* start = reinterpret_cast<int*>(smem_raw);  // [Nb + 1]
  int* list = start + Nb + 1;                     // [Na*K]
  int* wcount = list + Na * K;                    // [sort_warps][Nb]: per-warp counts, then cursors
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int bb = blockIdx.x;
  const int c0 = blockIdx.y * CC;
  const int E = Na * K;
  const int64_t eb = (int64_t)bb * E;
  // stable counting sort by receiver: sort warp w (of sort_warps <= nw, as
  // many as the shared memory holds count rows for) takes the contiguous
  // edge segment [w * seg, (w + 1) * seg), counts its receivers, and after a
  // prefix over (receiver, warp) places its edges in ascending edge order
  const int seg = (E + sort_warps - 1) / sort_warps;
  const bool sorter = warp < sort_warps;
  const int e_lo = sorter ? min(E, warp * seg) : E, e_hi = sorter ? min(E, e_lo + seg) : E;
  int* mycount = wcount + (sorter ? warp : 0) * Nb;
  if (sorter)
    for (int i = lane; i < Nb; i += 32) mycount[i] = 0;
  __syncwarp();
  auto key_of = [&](int e) -> int {
    const int64_t r = ridx[eb + e];
    return (rvalid[eb + e] && r >= 0 && r < Nb) ? (int)r : -1;
  };
  for (int base = e_lo; base < e_hi; base += 32) {
    const int e = base + lane;
    const int key = e < e_hi ? key_of(e) : -1;
    if (e < e_hi && key < 0 && rvalid[eb + e] && status) atomicOr(status, MN_STATUS_TOO_MANY_EDGES);
    const unsigned peers = __match_any_sync(MN_FULL_MASK, key);
    if (key >= 0 && lane == __ffs(peers) - 1) mycount[key] += __popc(peers);
    __syncwarp();
  }
  __syncthreads();
  // start[r] = edges of receivers < r; each warp's cursor for r begins after
  // the lower warps' edges into r
  for (int r = threadIdx.x; r < Nb; r += blockDim.x) {
    int tot = 0;
    for (int ww = 0; ww < sort_warps; ++ww) {
      const int cnt = wcount[ww * Nb + r];
      wcount[ww * Nb + r] = tot;
      tot += cnt;
    }
    start[r + 1] = tot;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    start[0] = 0;
    for (int i = 0; i < Nb; ++i) start[i + 1] += start[i];
  }
  __syncthreads();
  for (int base = e_lo; base < e_hi; base += 32) {
    const int e = base + lane;
    const int key = e < e_hi ? key_of(e) : -1;
    const unsigned peers = __match_any_sync(MN_FULL_MASK, key);
    const int rank = __popc(peers & ((1u << lane) - 1u));
    if (key >= 0) list[start[key] + mycount[key] + rank] = e;
    __syncwarp();
    if (key >= 0 && lane == __ffs(peers) - 1) mycount[key] += __popc(peers);
    __syncwarp();
  }
  __syncthreads();
  // gather, every (receiver, channel) sum in ascending edge order (the
  // reference's sequential scatter order: mul, then add, no fused
  // multiply-add)
  const ET* wb = w + eb;
  const ET* vb = v + (int64_t)bb * Na * C;
  const int c_end = min(C, c0 + CC);
  if (c_end - c0 <= 8) {
    // few channels (the masses and centres): a thread per receiver
    for (int r = threadIdx.x; r < Nb; r += blockDim.x) {
      const int j0 = start[r], j1 = start[r + 1];
      for (int c = c0; c < c_end; ++c) {
        float acc = 0.f;
        for (int j = j0; j < j1; ++j) {
          const int e = list[j];
          acc = __fadd_rn(acc, __fmul_rn(to_f32(wb[e]), to_f32(vb[(int64_t)(e / K) * C + c])));
        }
        out[((int64_t)bb * Nb + r) * C + c] = from_f32<ET>(acc);
      }
    }
    return;
  }
  // a lane accumulates up to four channels (32 apart) of one receiver; the
  // loads of four edges are in flight before their products are added
  for (int r = warp; r < Nb; r += nw) {
    const int j0 = start[r], j1 = start[r + 1];
    for (int cb = c0; cb < c_end; cb += 128) {
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      for (int j = j0; j < j1; j += 4) {
        float we[4], vv[4][4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const bool has = j + u < j1;
          const int e = list[has ? j + u : j0];
          we[u] = has ? to_f32(wb[e]) : 0.f;
          const ET* vrow = vb + (int64_t)(e / K) * C;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int c = cb + q * 32 + lane;
            vv[u][q] = (has && c < c_end) ? to_f32(vrow[c]) : 0.f;
          }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if (j + u >= j1) break;
#pragma unroll
          for (int q = 0; q < 4; ++q) acc[q] = __fadd_rn(acc[q], __fmul_rn(we[u], vv[u][q]));
        }
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int c = cb + q * 32 + lane;
        if (c < c_end) out[((int64_t)bb * Nb + r) * C + c] = from_f32<ET>(acc[q]);
      }
    }
  }
}

// Adjoint of the transport (dtem.py:962-973): a gather per donor, one warp
// per donor row.  G > 0: the donor's value row and its gradient row live in
// registers (G channel groups of 32 per lane, C <= 32 G), and every
// receiver row is read once for both the assignment's gradient (a dot
// product) and the values' gradient.  G == 0: any C, two passes.
// The same adjoint for narrow rows (C <= 8: masses, centres): one warp per
// donor row with a lane per slot (slots 32 apart loop), so every slot's
// receiver row is read at once; grad_w[k] = g[r_k] . v is the lane's own
// sum, and grad_v[c] = sum_k w_k g[r_k][c] one warp reduction per channel.
template <typename ET>
__global__ void __launch_bounds__(256) transport_adjoint_narrow_kernel(
    const ET* __restrict__ w, const ET* __restrict__ v, const int64_t* __restrict__ ridx,
    const uint8_t* __restrict__ rvalid, const ET* __restrict__ g, int B, int Na, int Nb, int K, int C,
    ET* __restrict__ grad_w, ET* __restrict__ grad_v) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= (int64_t)B * Na) return;
  const int bb = (int)(row / Na);
  float vr[8], gv[8];
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    vr[c] = c < C ? to_f32(v[row * C + c]) : 0.f;
    gv[c] = 0.f;
  }
  for (int k0 = 0; k0 < K; k0 += 32) {
    const int k = k0 + lane;
    float dot = 0.f;
    if (k < K) {
      const int64_t o = row * K + k;
      const int64_t s = ridx[o];
      if (rvalid[o] && s >= 0 && s < Nb) {
        const ET* grow = g + ((int64_t)bb * Nb + s) * C;
        const float wk = to_f32(w[o]);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          if (c < C) {
            const float gc = to_f32(grow[c]);
            dot = fmaf(gc, vr[c], dot);
            gv[c] = fmaf(wk, gc, gv[c]);
          }
        }
      }
      grad_w[o] = from_f32<ET>(dot);
    }
  }
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    if (c >= C) break;
    const float t = warp_sum(gv[c]);
    if (lane == 0) grad_v[row * C + c] = from_f32<ET>(t);
  }
}

template <typename ET, int G>
__global__ void __launch_bounds__(256) transport_adjoint_kernel(
    const ET* __restrict__ w, const ET* __restrict__ v, const int64_t* __restrict__ ridx,
    const uint8_t* __restrict__ rvalid, const ET* __restrict__ g, int B, int Na, int Nb, int K, int C,
    ET* __restrict__ grad_w, ET* __restrict__ grad_v) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= (int64_t)B * Na) return;
  const int bb = (int)(row / Na);
  const ET* vrow = v + row * C;
  if constexpr (G > 0) {
    float vr[G], gv[G];
#pragma unroll
    for (int q = 0; q < G; ++q) {
      const int c = q * 32 + lane;
      vr[q] = c < C ? to_f32(vrow[c]) : 0.f;
      gv[q] = 0.f;
    }
    for (int k = 0; k < K; ++k) {
      const int64_t o = row * K + k;
      const int64_t s = ridx[o];
      float dot = 0.f;
      if (rvalid[o] && s >= 0 && s < Nb) {
        const ET* grow = g + ((int64_t)bb * Nb + s) * C;
        const float wk = to_f32(w[o]);
        float gr[G];
#pragma unroll
        for (int q = 0; q < G; ++q) {
          const int c = q * 32 + lane;
          gr[q] = c < C ? to_f32(grow[c]) : 0.f;
        }
#pragma unroll
        for (int q = 0; q < G; ++q) {
          dot = fmaf(gr[q], vr[q], dot);
          gv[q] = fmaf(wk, gr[q], gv[q]);
        }
        dot = warp_sum(dot);
      }
      if (lane == 0) grad_w[o] = from_f32<ET>(dot);
    }
#pragma unroll
    for (int q = 0; q < G; ++q) {
      const int c = q * 32 + lane;
      if (c < C) grad_v[row * C + c] = from_f32<ET>(gv[q]);
    }
  } else {
    for (int k = 0; k < K; ++k) {
      const int64_t o = row * K + k;
      const int64_t s = ridx[o];
      float acc = 0.f;
      if (rvalid[o] && s >= 0 && s < Nb) {
        const ET* grow = g + ((int64_t)bb * Nb + s) * C;
        for (int c = lane; c < C; c += 32) acc = fmaf(to_f32(grow[c]), to_f32(vrow[c]), acc);
        acc = warp_sum(acc);
      }
      if (lane == 0) grad_w[o] = from_f32<ET>(acc);
    }
    for (int c = lane; c < C; c += 32) {
      float acc = 0.f;
      for (int k = 0; k < K; ++k) {
        const int64_t o = row * K + k;
        const int64_t s = ridx[o];
        if (rvalid[o] && s >= 0 && s < Nb)
          acc = fmaf(to_f32(w[o]), to_f32(g[((int64_t)bb * Nb + s) * C + c]), acc);
      }
      grad_v[row * C + c] = from_f32<ET>(acc);
    }
  }
}

// --------------------------------------------------------------------------
// ThreTopK and the soft-k-max select
// --------------------------------------------------------------------------
__global__ void __launch_bounds__(256) minmax_partials_kernel(const float* __restrict__ x, int64_t n,
                                                              float* __restrict__ partials) {
  __shared__ float red[64];
  float lo = INFINITY, hi = -INFINITY;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float v = x[i];
    lo = fminf(lo, v);
    hi = fmaxf(hi, v);
  }
  block_minmax(lo, hi, red);
  if (threadIdx.x == 0) {
    partials[2 * blockIdx.x] = lo;
    partials[2 * blockIdx.x + 1] = hi;
  }
}

__device__ __forceinline__ float reduce_range(const float* partials, int nparts, float* red, int* status) {
  float lo = INFINITY, hi = -INFINITY;
  for (int i = threadIdx.x; i < nparts; i += blockDim.x) {
    lo = fminf(lo, partials[2 * i]);
    hi = fmaxf(hi, partials[2 * i + 1]);
  }
  block_minmax(lo, hi, red);
  const float range = hi - lo;
  if (threadIdx.x == 0 && blockIdx.x == 0 && status && !(range > 0.f && range < INFINITY))
    atomicOr(status, MN_STATUS_DEGENERATE_RANGE);
  return range;
}

__global__ void __launch_bounds__(512) thre_topk_rows_kernel(const float* __restrict__ x, int n, int k,
                                                             float temperature, const float* partials,
                                                             int nparts, float* __restrict__ y, int* status) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ float red[64];
  const int np = next_pow2(n);
  RowScratch rs = carve_row_scratch(smem_raw, np);
  float* xrow = reinterpret_cast<float*>(smem_raw + row_scratch_bytes(np));
  const float range = reduce_range(partials, nparts, red, status);
  const float* xr = x + (int64_t)blockIdx.x * n;
  for (int i = threadIdx.x; i < n; i += blockDim.x) xrow[i] = xr[i] / range * temperature;
  __syncthreads();
  const float lam = thre_topk_lambda(xrow, n, np, k, rs);
  for (int i = threadIdx.x; i < n; i += blockDim.x) y[(int64_t)blockIdx.x * n + i] = thre_topk_map(xrow[i], lam);
}

// Gradient of ThreTopK with respect to x: the closed form of the reference's
// autograd through thetopk.py:4-43.  Per row (one CTA), after
// thre_topk_lambda has left the sorted row and its scans in rs and returned
// lambda and the bracket b:
//   dx~_i = f'(d_i) g_i + [s(i) <= b] dlse1 e^{x~_i - lse1_b}
//           - [s(i) > b] dL e^{-x~_i - lse2_b}
// with s(i) the place of i in the stable ascending sort, dlambda =
// -sum_i f'(d_i) g_i, dL the path through |term_b|, dlse1 = dlambda + dL.
// Writes gx[i] = dx~_i T / R and returns (in every thread) the row's share
// of dR = -sum_i dx~_i x_i T / R^2, which thre_topk_grad_range_kernel adds
// to the maximum and subtracts from the minimum elements.
// xrow: the row's scaled values x~ (shared); xr: its unscaled values; g:
// the upstream gradient (readable by every thread).
__device__ float thre_topk_row_grad(const float* xrow, const float* xr, const float* g, int n, int k, float lam,
                                    int b, float range, float temperature, const RowScratch& rs, float* red,
                                    float* __restrict__ gx) {
  const float xs_b = rs.xs[b], lse1_b = rs.lse1[b];
  const float lse2_b = b + 1 < n ? (float)(-(double)rs.xs[0] + log(rs.dbuf[n - 2 - b])) : -INFINITY;
  const float km = (float)(k - (n - 1 - b));
  const float el = expf(lse1_b + lse2_b);
  const float term = sqrtf(km * km + el) + km;
  auto fprime = [&](float v) {
    const float dv = v - lam;
    return dv > 0.f ? 0.5f * expf(-dv) : 0.5f * expf(dv);
  };
  float sdd = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) sdd += g[i] * fprime(xrow[i]);
  sdd = block_sum(sdd, red);
  const float dlam = -sdd;
  const float sgn = term > 0.f ? 1.f : (term < 0.f ? -1.f : 0.f);
  const float dterm = -dlam / (fabsf(term) + 1e-8f) * sgn;
  const float dl = el > 0.f ? dterm * 0.5f / sqrtf(km * km + el) * el : 0.f;
  const float dlse1 = dlam + dl;
  const float inv_r = temperature / range;
  // elements equal to xs_b take their side from their place in the stable
  // sort: below_b values lie under xs_b, and ties rank by index after them
  int below_b = 0;
  for (int hi = b; below_b < hi;) {
    const int mid = (below_b + hi) >> 1;
    if (rs.xs[mid] < xs_b) below_b = mid + 1;
    else hi = mid;
  }
  float part = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = xrow[i];
    float dxt = g[i] * fprime(v);
    bool low = v < xs_b;
    if (v == xs_b) {
      int pos = below_b;
      for (int j = 0; j < i; ++j) pos += xrow[j] == xs_b;
      low = pos <= b;
    }
    if (low) dxt += dlse1 * expf(v - lse1_b);
    else if (b + 1 < n) dxt -= dl * expf(-v - lse2_b);
    gx[i] = dxt * inv_r;
    part += dxt * xr[i];
  }
  part = block_sum(part, red);
  return -part * inv_r / range;
}

__global__ void __launch_bounds__(512) thre_topk_grad_rows_kernel(const float* __restrict__ x,
                                                                  const float* __restrict__ gy, int n, int k,
                                                                  float temperature, const float* partials,
                                                                  int nparts, float* __restrict__ gx,
                                                                  float* __restrict__ rpart, int* status) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ float red[64];
  const int np = next_pow2(n);
  RowScratch rs = carve_row_scratch(smem_raw, np);
  float* xrow = reinterpret_cast<float*>(smem_raw + row_scratch_bytes(np));
  const float range = reduce_range(partials, nparts, red, status);
  const int64_t row = blockIdx.x;
  const float* xr = x + row * n;
  for (int i = threadIdx.x; i < n; i += blockDim.x) xrow[i] = xr[i] / range * temperature;
  __syncthreads();
  int b = 0;
  const float lam = thre_topk_lambda(xrow, n, np, k, rs, &b);
  const float part = thre_topk_row_grad(xrow, xr, gy + row * n, n, k, lam, b, range, temperature, rs, red,
                                        gx + row * n);
  if (threadIdx.x == 0) rpart[row] = part;
}

// The range's share of the ThreTopK gradient: dR (the sum of the rows'
// partials) to every maximum element and -dR to every minimum element, split
// evenly over ties as the reference's autograd splits max() / min().
__global__ void __launch_bounds__(1024) thre_topk_grad_range_kernel(const float* __restrict__ x, int64_t total,
                                                                   const float* __restrict__ rpart, int rows,
                                                                   const float* partials, int nparts,
                                                                   float* __restrict__ gx) {
  __shared__ float red[64];
  __shared__ int cnt[2];
  float lo = INFINITY, hi = -INFINITY;
  for (int i = threadIdx.x; i < nparts; i += blockDim.x) {
    lo = fminf(lo, partials[2 * i]);
    hi = fmaxf(hi, partials[2 * i + 1]);
  }
  block_minmax(lo, hi, red);
  float dr = 0.f;
  for (int r = threadIdx.x; r < rows; r += blockDim.x) dr += rpart[r];
  dr = block_sum(dr, red);
  if (threadIdx.x == 0) cnt[0] = cnt[1] = 0;
  __syncthreads();
  int nmax = 0, nmin = 0;
  for (int64_t i = threadIdx.x; i < total; i += blockDim.x) {
    nmax += x[i] == hi;
    nmin += x[i] == lo;
  }
  atomicAdd(&cnt[0], nmax);  // integer counts: order-independent
  atomicAdd(&cnt[1], nmin);
  __syncthreads();
  const float add_max = dr / (float)max(cnt[0], 1), add_min = dr / (float)max(cnt[1], 1);
  for (int64_t i = threadIdx.x; i < total; i += blockDim.x) {
    if (x[i] == hi) gx[i] += add_max;
    if (x[i] == lo) gx[i] -= add_min;
  }
}

// Row energies of the masked scores (dtem.py:1557-1567): one warp per row.
__global__ void __launch_bounds__(256) select_energy_kernel(const float* __restrict__ scores,
                                                            const uint8_t* __restrict__ allowed, int rows,
                                                            int K, float tau1, float* __restrict__ energy,
                                                            int* __restrict__ valid_count, int Na) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float* s = scores + row * K;
  const uint8_t* al = allowed + row * K;
  float m = -INFINITY;
  for (int k = lane; k < K; k += 32)
    if (al[k]) m = fmaxf(m, s[k] / tau1);
  m = warp_max(m);
  float e = 0.f;
  if (m != -INFINITY) {
    float sum = 0.f;
    for (int k = lane; k < K; k += 32)
      if (al[k]) sum += expf(s[k] / tau1 - m);
    sum = warp_sum(sum);
    e = expf(logf(sum) + m);
  }
  if (lane == 0) {
    energy[row] = e;
    if (valid_count && m != -INFINITY) atomicAdd(&valid_count[row / Na], 1);
  }
}

// The select's per-image threshold: one CTA per image computes lambda of
// ThreTopK over the image's row energies (thetopk.py:4-43) and flags an
// infeasible budget; select_rows_kernel then forms every donor row.
__global__ void __launch_bounds__(512) select_lambda_kernel(int Na, int k, float tau2,
                                                            const float* __restrict__ energy,
                                                            const int* __restrict__ valid_count,
                                                            const float* partials, int nparts,
                                                            float* __restrict__ lam_out, int* status) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ float red[64];
  const int np = next_pow2(Na);
  RowScratch rs = carve_row_scratch(smem_raw, np);
  float* xrow = reinterpret_cast<float*>(smem_raw + row_scratch_bytes(np));
  const int bb = blockIdx.x;
  if (threadIdx.x == 0 && valid_count[bb] < k && status) atomicOr(status, MN_STATUS_INFEASIBLE_BUDGET);
  const float range = reduce_range(partials, nparts, red, status);
  const float* e = energy + (int64_t)bb * Na;
  for (int i = threadIdx.x; i < Na; i += blockDim.x) xrow[i] = e[i] / range * tau2;
  __syncthreads();
  const float lam = thre_topk_lambda(xrow, Na, np, k, rs);
  if (threadIdx.x == 0) lam_out[bb] = lam;
}

// Every donor row of the select (dtem.py:1557-1579), one thread per row:
// the masked softmax x the row's k-hot y = map(E / range * tau2, lambda),
// then the clamp-normalise.  The CTA's 256 rows of scores and mask are
// staged in shared memory with coalesced loads (a row is K values apart per
// thread), and the assignment leaves the same way.
__global__ void __launch_bounds__(256) select_rows_kernel(const float* __restrict__ scores,
                                                          const uint8_t* __restrict__ allowed, int rows, int Na,
                                                          int K, float tau1, float tau2,
                                                          const float* __restrict__ energy,
                                                          const float* partials, int nparts,
                                                          const float* __restrict__ lam_in,
                                                          float* __restrict__ assign) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ float red[64];
  float* sbuf = reinterpret_cast<float*>(smem_raw);                        // [256 * K]
  uint8_t* abuf = reinterpret_cast<uint8_t*>(sbuf + (size_t)blockDim.x * K);  // [256 * K]
  const float range = reduce_range(partials, nparts, red, nullptr);
  const int64_t row0 = (int64_t)blockIdx.x * blockDim.x;
  const int nrows = (int)(rows - row0 < (int64_t)blockDim.x ? rows - row0 : (int64_t)blockDim.x);
  const int64_t base = row0 * K;
  for (int i = threadIdx.x; i < nrows * K; i += blockDim.x) {
    sbuf[i] = scores[base + i];
    abuf[i] = allowed[base + i];
  }
  __syncthreads();
  const int r = threadIdx.x;
  if (r < nrows) {
    const int64_t row = row0 + r;
    const float* s = sbuf + r * K;
    const uint8_t* al = abuf + r * K;
    float* out = sbuf + r * K;  // the row's assignment replaces its scores
    float m = -INFINITY;
    for (int c = 0; c < K; ++c)
      if (al[c]) m = fmaxf(m, s[c] / tau1);
    if (m == -INFINITY) {
      for (int c = 0; c < K; ++c) out[c] = 0.f;
    } else {
      const float y = thre_topk_map(energy[row] / range * tau2, lam_in[row / Na]);
      float sum = 0.f;
      for (int c = 0; c < K; ++c)
        if (al[c]) sum += expf(s[c] / tau1 - m);
      const float inv = 1.0f / sum;
      float ks = 0.f;
      for (int c = 0; c < K; ++c) {
        const float kh = al[c] ? (expf(s[c] / tau1 - m) * inv) * y : 0.f;
        out[c] = kh;
        ks += kh;
      }
      const float tmp = fmaxf(ks - 1.0f, 0.0f) + 1.0f;
      for (int c = 0; c < K; ++c) out[c] = out[c] / tmp;
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < nrows * K; i += blockDim.x) assign[base + i] = sbuf[i];
}

// Select backward, part 1 (one CTA per batch row): recompute lambda over
// the row energies, then per donor row the masked softmax p, y = ThreTopK
// (times the valid-row flag) and t = max(sum_j p_j y - 1, 0) + 1 (detached
// in the reference), the upstream gradient of y, dy = sum_j G_j p_j / t,
// and through thre_topk_row_grad the energies' gradient (before the range
// share) and the batch row's share of dR.  y and t go to the workspace for
// part 2.
__global__ void __launch_bounds__(512) select_grad_rows_kernel(const float* __restrict__ scores,
                                                               const uint8_t* __restrict__ allowed,
                                                               const float* __restrict__ grad_assign, int Na,
                                                               int K, int k, float tau1, float tau2,
                                                               const float* __restrict__ energy,
                                                               const float* partials, int nparts,
                                                               float* __restrict__ yrow_out,
                                                               float* __restrict__ trow_out,
                                                               float* __restrict__ grad_energy,
                                                               float* __restrict__ rpart, int* status) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ float red[64];
  const int np = next_pow2(Na);
  RowScratch rs = carve_row_scratch(smem_raw, np);
  float* xrow = reinterpret_cast<float*>(smem_raw + row_scratch_bytes(np));
  float* dy = xrow + Na;
  const int bb = blockIdx.x;
  const float range = reduce_range(partials, nparts, red, status);
  const float* e = energy + (int64_t)bb * Na;
  for (int i = threadIdx.x; i < Na; i += blockDim.x) xrow[i] = e[i] / range * tau2;
  __syncthreads();
  int b = 0;
  const float lam = thre_topk_lambda(xrow, Na, np, k, rs, &b);
  for (int d = threadIdx.x; d < Na; d += blockDim.x) {
    const int64_t row = (int64_t)bb * Na + d;
    const float* s = scores + row * K;
    const uint8_t* al = allowed + row * K;
    const float* g = grad_assign + row * K;
    float m = -INFINITY;
    for (int c = 0; c < K; ++c)
      if (al[c]) m = fmaxf(m, s[c] / tau1);
    float y = 0.f, t = 1.f, gy = 0.f;
    if (m != -INFINITY) {
      y = thre_topk_map(xrow[d], lam);
      float sum = 0.f;
      for (int c = 0; c < K; ++c)
        if (al[c]) sum += expf(s[c] / tau1 - m);
      const float inv = 1.0f / sum;
      float ks = 0.f, gp = 0.f;
      for (int c = 0; c < K; ++c) {
        if (!al[c]) continue;
        const float pc = expf(s[c] / tau1 - m) * inv;
        ks += pc * y;
        gp += g[c] * pc;
      }
      t = fmaxf(ks - 1.0f, 0.0f) + 1.0f;
      gy = gp / t;
    }
    dy[d] = gy;
    yrow_out[row] = y;
    trow_out[row] = t;
  }
  __syncthreads();
  const float part = thre_topk_row_grad(xrow, e, dy, Na, k, lam, b, range, tau2, rs, red,
                                        grad_energy + (int64_t)bb * Na);
  if (threadIdx.x == 0) rpart[bb] = part;
}

// Select backward, part 2 (one warp per donor row): with dp_j = G_j y / t,
// dscores_j = p_j (dp_j - sum_l dp_l p_l + dE E) / tau1 on allowed slots of
// valid rows (the softmax's and the logsumexp's backward), zero elsewhere.
__global__ void __launch_bounds__(256) select_grad_out_kernel(const float* __restrict__ scores,
                                                              const uint8_t* __restrict__ allowed,
                                                              const float* __restrict__ grad_assign, int rows,
                                                              int K, float tau1, const float* __restrict__ energy,
                                                              const float* __restrict__ grad_energy,
                                                              const float* __restrict__ yrow,
                                                              const float* __restrict__ trow,
                                                              float* __restrict__ grad_scores) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float* s = scores + row * K;
  const uint8_t* al = allowed + row * K;
  const float* g = grad_assign + row * K;
  float* out = grad_scores + row * K;
  float m = -INFINITY;
  for (int c = lane; c < K; c += 32)
    if (al[c]) m = fmaxf(m, s[c] / tau1);
  m = warp_max(m);
  if (m == -INFINITY) {
    for (int c = lane; c < K; c += 32) out[c] = 0.f;
    return;
  }
  float sum = 0.f;
  for (int c = lane; c < K; c += 32)
    if (al[c]) sum += expf(s[c] / tau1 - m);
  const float inv = 1.0f / warp_sum(sum);
  const float scale = yrow[row] / trow[row];
  float inner = 0.f;
  for (int c = lane; c < K; c += 32)
    if (al[c]) inner += g[c] * scale * (expf(s[c] / tau1 - m) * inv);
  inner = warp_sum(inner);
  const float dlse = grad_energy[row] * energy[row];
  for (int c = lane; c < K; c += 32) {
    float v = 0.f;
    if (al[c]) {
      const float pc = expf(s[c] / tau1 - m) * inv;
      v = pc * (g[c] * scale - inner + dlse) / tau1;
    }
    out[c] = v;
  }
}

// Transpose of the carrier gather, one pass over the output: a CTA owns
// kScatterRows patch rows of one image, maps each to its carrier through an
// inverse table of the image's carrier indices (built in shared memory; if a
// patch is listed twice the later carrier wins) and writes every row once,
// the carrier's features or zeros, with 16-byte stores when the rows allow.
constexpr int kScatterRows = 64;

template <typename ET>
__global__ void __launch_bounds__(256) carrier_scatter_kernel(const ET* __restrict__ topk_x,
                                                              const int64_t* __restrict__ idx, int k, int P,
                                                              int C, ET* __restrict__ out) {
  __shared__ int inv[kScatterRows];
  const int bb = blockIdx.y;
  const int p0 = blockIdx.x * kScatterRows;
  const int nrows = min(kScatterRows, P - p0);
  for (int r = threadIdx.x; r < nrows; r += blockDim.x) inv[r] = -1;
  __syncthreads();
  const int64_t* ib = idx + (int64_t)bb * k;
  for (int i = threadIdx.x; i < k; i += blockDim.x) {
    const int64_t p = ib[i];
    if (p >= p0 && p < p0 + nrows) atomicMax(&inv[p - p0], i);
  }
  __syncthreads();
  const ET* src_b = topk_x + ((int64_t)bb * (k + 1) + 1) * C;
  ET* dst_b = out + ((int64_t)bb * P + p0) * C;
  const bool vec = (C * (int)sizeof(ET)) % 16 == 0 && (reinterpret_cast<uintptr_t>(topk_x) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(out) & 15) == 0;
  if (vec) {
    const int vpr = C * (int)sizeof(ET) / 16;  // 16-byte vectors per row
    for (int e = threadIdx.x; e < nrows * vpr; e += blockDim.x) {
      const int r = e / vpr, v = e % vpr;
      const int i = inv[r];
      const uint4 val = i >= 0 ? reinterpret_cast<const uint4*>(src_b + (int64_t)i * C)[v] : make_uint4(0, 0, 0, 0);
      reinterpret_cast<uint4*>(dst_b + (int64_t)r * C)[v] = val;
    }
  } else {
    for (int e = threadIdx.x; e < nrows * C; e += blockDim.x) {
      const int r = e / C, c = e % C;
      const int i = inv[r];
      dst_b[(int64_t)r * C + c] = i >= 0 ? src_b[(int64_t)i * C + c] : from_f32<ET>(0.f);
    }
  }
}

template <typename F>
static int dispatch_dtype(int dtype, F&& f) {
  if (dtype == MN_F32) { f(float{}); return MN_OK; }
  if (dtype == MN_F16) { f(__half{}); return MN_OK; }
  if (dtype == MN_BF16) { f(__nv_bfloat16{}); return MN_OK; }
  return MN_ERR_ARG;
}

static int launch_status() { return cudaGetLastError() == cudaSuccess ? MN_OK : MN_ERR_LAUNCH; }

}  // namespace mn

using namespace mn;

extern "C" int mn_sparse_spatial_score(int batch, int num_donors, int num_receivers, int num_patches, int k,
                                       int channels, int dtype, const void* a, const void* b,
                                       const int64_t* neighbor_indices, const uint8_t* neighbor_valid,
                                       const int64_t* donor_patch, const int64_t* receiver_patch, void* scores,
                                       int64_t* receiver_indices, uint8_t* receiver_valid, void* stream) {
  if (batch < 0 || num_donors < 0 || num_receivers <= 0 || num_patches <= 0 || k <= 0 || channels <= 0)
    return MN_ERR_ARG;
  if ((int64_t)batch * num_donors == 0) return MN_OK;
  if (!a || !b || !neighbor_indices || !neighbor_valid || !donor_patch || !receiver_patch || !scores ||
      !receiver_indices || !receiver_valid)
    return MN_ERR_ARG;
  cudaGetLastError();
  const int64_t rows = (int64_t)batch * num_donors;
  const dim3 grid((unsigned)((rows + 7) / 8));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int rc = dispatch_dtype(dtype, [&](auto tag) {
    using ET = decltype(tag);
    const bool quad = (channels * (int)sizeof(ET)) % 64 == 0 && (reinterpret_cast<uintptr_t>(a) & 15) == 0 &&
                      (reinterpret_cast<uintptr_t>(b) & 15) == 0;
    auto kern = quad ? sparse_score_kernel<ET, true> : sparse_score_kernel<ET, false>;
    kern<<<grid, 256, 0, st>>>(static_cast<const ET*>(a), static_cast<const ET*>(b), neighbor_indices, neighbor_valid,
                               donor_patch, receiver_patch, batch, num_donors, num_receivers, num_patches, k, channels,
                               static_cast<ET*>(scores), receiver_indices, receiver_valid);
  });
  return rc != MN_OK ? rc : launch_status();
}

extern "C" int mn_sparse_neighbor_dot(int batch, int num_donors, int num_receivers, int k, int channels,
                                      int dtype, const void* a, const void* b, const int64_t* receiver_indices,
                                      const uint8_t* receiver_valid, void* scores, void* stream) {
  if (batch < 0 || num_donors < 0 || num_receivers <= 0 || k <= 0 || channels <= 0) return MN_ERR_ARG;
  if ((int64_t)batch * num_donors == 0) return MN_OK;
  if (!a || !b || !receiver_indices || !receiver_valid || !scores) return MN_ERR_ARG;
  cudaGetLastError();
  const int64_t rows = (int64_t)batch * num_donors;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int rc = dispatch_dtype(dtype, [&](auto tag) {
    using ET = decltype(tag);
    const bool quad = (channels * (int)sizeof(ET)) % 64 == 0 && (reinterpret_cast<uintptr_t>(a) & 15) == 0 &&
                      (reinterpret_cast<uintptr_t>(b) & 15) == 0;
    auto kern = quad ? neighbor_dot_kernel<ET, true> : neighbor_dot_kernel<ET, false>;
    kern<<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(
        static_cast<const ET*>(a), static_cast<const ET*>(b), receiver_indices, receiver_valid, batch,
        num_donors, num_receivers, k, channels, static_cast<ET*>(scores));
  });
  return rc != MN_OK ? rc : launch_status();
}

extern "C" int mn_sparse_weighted_transport(int batch, int num_donors, int num_receivers, int k, int channels,
                                            int dtype, const void* assignment, const void* values,
                                            const int64_t* receiver_indices, const uint8_t* receiver_valid,
                                            void* out, int* status, void* stream) {
  if (batch < 0 || num_donors < 0 || num_receivers <= 0 || k <= 0 || channels <= 0) return MN_ERR_ARG;
  if (batch == 0) return MN_OK;
  if (!out) return MN_ERR_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t elem = dtype == MN_F32 ? 4 : 2;
  cudaGetLastError();
  if (num_donors == 0) {
    cudaMemsetAsync(out, 0, (size_t)batch * num_receivers * channels * elem, st);
    return launch_status();
  }
  if (!assignment || !values || !receiver_indices || !receiver_valid) return MN_ERR_ARG;
  // edge starts, the edge list and up to 16 sort warps' per-receiver counts
  const size_t base_ints = (size_t)num_receivers + 1 + (size_t)num_donors * k;
  const size_t cap_ints = 200 * 1024 / sizeof(int);
  if (base_ints + num_receivers > cap_ints) return MN_ERR_UNSUPPORTED;
  const int sort_warps = (int)std::min<size_t>(16, (cap_ints - base_ints) / num_receivers);
  const size_t smem = (base_ints + (size_t)sort_warps * num_receivers) * sizeof(int);
  const int CC = 128;
  const dim3 grid(batch, (channels + CC - 1) / CC);
  int rc = dispatch_dtype(dtype, [&](auto tag) {
    using ET = decltype(tag);
    if (!ensure_smem(transport_kernel<ET>, smem)) return;  // reported by launch_status below
    transport_kernel<ET><<<grid, 512, smem, st>>>(static_cast<const ET*>(assignment), static_cast<const ET*>(values),
                                                  receiver_indices, receiver_valid, num_donors, num_receivers, k,
                                                  channels, CC, sort_warps, static_cast<ET*>(out), status);
  });
  return rc != MN_OK ? rc : launch_status();
}

extern "C" int mn_sparse_transport_adjoint(int batch, int num_donors, int num_receivers, int k, int channels,
                                           int dtype, const void* assignment, const void* values,
                                           const int64_t* receiver_indices, const uint8_t* receiver_valid,
                                           const void* grad_out, void* grad_assignment, void* grad_values,
                                           void* stream) {
  if (batch < 0 || num_donors < 0 || num_receivers <= 0 || k <= 0 || channels <= 0) return MN_ERR_ARG;
  if ((int64_t)batch * num_donors == 0) return MN_OK;
  if (!assignment || !values || !receiver_indices || !receiver_valid || !grad_out || !grad_assignment ||
      !grad_values)
    return MN_ERR_ARG;
  cudaGetLastError();
  const int64_t rows = (int64_t)batch * num_donors;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int rc = dispatch_dtype(dtype, [&](auto tag) {
    using ET = decltype(tag);
    auto launch = [&](auto kern) {
      kern<<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(
          static_cast<const ET*>(assignment), static_cast<const ET*>(values), receiver_indices, receiver_valid,
          static_cast<const ET*>(grad_out), batch, num_donors, num_receivers, k, channels,
          static_cast<ET*>(grad_assignment), static_cast<ET*>(grad_values));
    };
    const int groups = (channels + 31) / 32;
    if (channels <= 8) launch(transport_adjoint_narrow_kernel<ET>);
    else if (groups <= 1) launch(transport_adjoint_kernel<ET, 1>);
    else if (groups <= 2) launch(transport_adjoint_kernel<ET, 2>);
    else if (groups <= 4) launch(transport_adjoint_kernel<ET, 4>);
    else if (groups <= 8) launch(transport_adjoint_kernel<ET, 8>);
    else if (groups <= 12) launch(transport_adjoint_kernel<ET, 12>);
    else if (groups <= 16) launch(transport_adjoint_kernel<ET, 16>);
    else launch(transport_adjoint_kernel<ET, 0>);
  });
  return rc != MN_OK ? rc : launch_status();
}

static int thre_topk_parts(int64_t n) { return (int)std::min<int64_t>(1024, std::max<int64_t>(1, (n + 2047) / 2048)); }

extern "C" size_t mn_thre_topk_workspace_bytes(int rows, int n) {
  if (rows <= 0 || n <= 0) return 0;
  return (size_t)thre_topk_parts((int64_t)rows * n) * 2 * sizeof(float);
}

extern "C" int mn_thre_topk(int rows, int n, const float* x, int k, float temperature, float* y,
                            void* workspace, size_t workspace_bytes, int* status, void* stream) {
  if (rows <= 0 || n <= 0 || !x || !y || !workspace) return MN_ERR_ARG;
  if (n > 4096) return MN_ERR_UNSUPPORTED;
  if (workspace_bytes < mn_thre_topk_workspace_bytes(rows, n)) return MN_ERR_WORKSPACE;
  cudaGetLastError();
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int parts = thre_topk_parts((int64_t)rows * n);
  float* partials = static_cast<float*>(workspace);
  const int np = next_pow2(n);
  const size_t smem = row_scratch_bytes(np) + (size_t)n * sizeof(float);
  if (!ensure_smem(thre_topk_rows_kernel, smem)) return MN_ERR_LAUNCH;
  minmax_partials_kernel<<<parts, 256, 0, st>>>(x, (int64_t)rows * n, partials);
  thre_topk_rows_kernel<<<rows, 512, smem, st>>>(x, n, k, temperature, partials, parts, y, status);
  return launch_status();
}

extern "C" size_t mn_thre_topk_backward_workspace_bytes(int rows, int n) {
  if (rows <= 0 || n <= 0) return 0;
  return mn_thre_topk_workspace_bytes(rows, n) + (size_t)rows * sizeof(float);
}

extern "C" int mn_thre_topk_backward(int rows, int n, const float* x, int k, float temperature, const float* grad_y,
                                     float* grad_x, void* workspace, size_t workspace_bytes, int* status,
                                     void* stream) {
  if (rows <= 0 || n <= 0 || !x || !grad_y || !grad_x || !workspace) return MN_ERR_ARG;
  if (n > 4096) return MN_ERR_UNSUPPORTED;
  if (workspace_bytes < mn_thre_topk_backward_workspace_bytes(rows, n)) return MN_ERR_WORKSPACE;
  cudaGetLastError();
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int parts = thre_topk_parts((int64_t)rows * n);
  float* partials = static_cast<float*>(workspace);
  float* rpart = partials + 2 * parts;
  const int np = next_pow2(n);
  const size_t smem = row_scratch_bytes(np) + (size_t)n * sizeof(float);
  if (!ensure_smem(thre_topk_grad_rows_kernel, smem)) return MN_ERR_LAUNCH;
  minmax_partials_kernel<<<parts, 256, 0, st>>>(x, (int64_t)rows * n, partials);
  thre_topk_grad_rows_kernel<<<rows, 512, smem, st>>>(x, grad_y, n, k, temperature, partials, parts, grad_x, rpart,
                                                      status);
  thre_topk_grad_range_kernel<<<1, 1024, 0, st>>>(x, (int64_t)rows * n, rpart, rows, partials, parts, grad_x);
  return launch_status();
}

extern "C" size_t mn_dtem_select_workspace_bytes(int batch, int num_donors) {
  if (batch <= 0 || num_donors <= 0) return 0;
  const int64_t rows = (int64_t)batch * num_donors;
  return (size_t)rows * sizeof(float) + (size_t)batch * sizeof(int) +
         (size_t)thre_topk_parts(rows) * 2 * sizeof(float) + (size_t)batch * sizeof(float) + 64;
}

// The select after the row energies and their min/max partials: lambda per
// image, then every donor row.
static void launch_select(int batch, int num_donors, int k_slots, const float* scores, const uint8_t* allowed, int k,
                          float tau1, float tau2, const float* energy, const int* counts, const float* partials,
                          int parts, float* lam, size_t smem, float* assignment, int* status, cudaStream_t st) {
  const int64_t rows = (int64_t)batch * num_donors;
  select_lambda_kernel<<<batch, 512, smem, st>>>(num_donors, k, tau2, energy, counts, partials, parts, lam, status);
  select_rows_kernel<<<(unsigned)((rows + 255) / 256), 256, (size_t)256 * k_slots * 5, st>>>(
      scores, allowed, (int)rows, num_donors, k_slots, tau1, tau2, energy, partials, parts, lam, assignment);
}

extern "C" int mn_dtem_select(int batch, int num_donors, int k_slots, const float* scores, const uint8_t* allowed,
                              int k, float tau1, float tau2, float* assignment, void* workspace,
                              size_t workspace_bytes, int* status, void* stream) {
  if (batch <= 0 || num_donors <= 0 || k_slots <= 0 || !scores || !allowed || !assignment || !workspace)
    return MN_ERR_ARG;
  if (num_donors > 4096) return MN_ERR_UNSUPPORTED;
  if (workspace_bytes < mn_dtem_select_workspace_bytes(batch, num_donors)) return MN_ERR_WORKSPACE;
  cudaGetLastError();
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t rows = (int64_t)batch * num_donors;
  float* energy = static_cast<float*>(workspace);
  int* counts = reinterpret_cast<int*>(energy + rows);
  float* partials = reinterpret_cast<float*>(counts + batch);
  const int parts = thre_topk_parts(rows);
  float* lam = partials + 2 * parts;
  const int np = next_pow2(num_donors);
  const size_t smem = row_scratch_bytes(np) + (size_t)num_donors * sizeof(float);
  if (k_slots > 160) return MN_ERR_UNSUPPORTED;  // the row kernel stages 256 rows of K slots
  if (!ensure_smem(select_lambda_kernel, smem) || !ensure_smem(select_rows_kernel, (size_t)256 * k_slots * 5))
    return MN_ERR_LAUNCH;
  cudaMemsetAsync(counts, 0, (size_t)batch * sizeof(int), st);
  select_energy_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(scores, allowed, (int)rows, k_slots, tau1,
                                                                   energy, counts, num_donors);
  minmax_partials_kernel<<<parts, 256, 0, st>>>(energy, rows, partials);
  launch_select(batch, num_donors, k_slots, scores, allowed, k, tau1, tau2, energy, counts, partials, parts, lam, smem,
                assignment, status, st);
  return launch_status();
}

extern "C" size_t mn_dtem_select_backward_workspace_bytes(int batch, int num_donors) {
  if (batch <= 0 || num_donors <= 0) return 0;
  const int64_t rows = (int64_t)batch * num_donors;
  return (size_t)rows * 4 * sizeof(float) + (size_t)thre_topk_parts(rows) * 2 * sizeof(float) +
         (size_t)batch * sizeof(float) + 64;
}

extern "C" int mn_dtem_select_backward(int batch, int num_donors, int k_slots, const float* scores,
                                       const uint8_t* allowed, int k, float tau1, float tau2,
                                       const float* grad_assignment, float* grad_scores, void* workspace,
                                       size_t workspace_bytes, int* status, void* stream) {
  if (batch <= 0 || num_donors <= 0 || k_slots <= 0 || !scores || !allowed || !grad_assignment || !grad_scores ||
      !workspace)
    return MN_ERR_ARG;
  if (num_donors > 4096) return MN_ERR_UNSUPPORTED;
  if (workspace_bytes < mn_dtem_select_backward_workspace_bytes(batch, num_donors)) return MN_ERR_WORKSPACE;
  cudaGetLastError();
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t rows = (int64_t)batch * num_donors;
  const int parts = thre_topk_parts(rows);
  float* energy = static_cast<float*>(workspace);
  float* grad_energy = energy + rows;
  float* yrow = grad_energy + rows;
  float* trow = yrow + rows;
  float* partials = trow + rows;
  float* rpart = partials + 2 * parts;
  const int np = next_pow2(num_donors);
  const size_t smem = row_scratch_bytes(np) + (size_t)2 * num_donors * sizeof(float);
  if (!ensure_smem(select_grad_rows_kernel, smem)) return MN_ERR_LAUNCH;
  select_energy_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(scores, allowed, (int)rows, k_slots, tau1,
                                                                   energy, nullptr, num_donors);
  minmax_partials_kernel<<<parts, 256, 0, st>>>(energy, rows, partials);
  select_grad_rows_kernel<<<batch, 512, smem, st>>>(scores, allowed, grad_assignment, num_donors, k_slots, k, tau1,
                                                    tau2, energy, partials, parts, yrow, trow, grad_energy, rpart,
                                                    status);
  thre_topk_grad_range_kernel<<<1, 1024, 0, st>>>(energy, rows, rpart, batch, partials, parts, grad_energy);
  select_grad_out_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(scores, allowed, grad_assignment, (int)rows,
                                                                     k_slots, tau1, energy, grad_energy, yrow, trow,
                                                                     grad_scores);
  return launch_status();
}

extern "C" int mn_carrier_scatter(int batch, int k, int num_patches, int channels, int dtype, const void* topk_x,
                                  const int64_t* topk_idx, void* out, void* stream) {
  if (batch < 0 || k < 0 || num_patches <= 0 || channels <= 0 || !out) return MN_ERR_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t elem = dtype == MN_F32 ? 4 : 2;
  cudaGetLastError();
  if (batch == 0) return launch_status();
  if (k == 0) {
    cudaMemsetAsync(out, 0, (size_t)batch * num_patches * channels * elem, st);
    return launch_status();
  }
  if (!topk_x || !topk_idx) return MN_ERR_ARG;
  if (batch > 65535) return MN_ERR_UNSUPPORTED;
  const dim3 grid((unsigned)((num_patches + kScatterRows - 1) / kScatterRows), (unsigned)batch);
  int rc = dispatch_dtype(dtype, [&](auto tag) {
    using ET = decltype(tag);
    carrier_scatter_kernel<ET><<<grid, 256, 0, st>>>(static_cast<const ET*>(topk_x), topk_idx, k, num_patches,
                                                     channels, static_cast<ET*>(out));
  });
  return rc != MN_OK ? rc : launch_status();
}

// ---------------------------------------------------------------------------
// mn_dtem_select_noalloc: the soft-k-max select for callers that cannot
// allocate device memory.  Some callers have no device allocator to draw on
// (a host application or language binding that hands the library raw
// pointers but owns no CUDA memory pool), and some must not call cudaMalloc
// at all (a serving loop that cannot afford the implicit device
// synchronisation and unpredictable latency of an allocation, or a process
// whose device memory is already carved up by another runtime).  This
// variant keeps its scratch (row energies, per-batch valid-row counts,
// energy min/max partials, per-image thresholds) in a fixed array compiled
// into the library, so the caller passes only inputs and outputs.
//
// The array holds at most kNoAllocMaxRows donor rows (batch * num_donors)
// and kNoAllocMaxBatch batch rows; larger calls are rejected with
// MN_ERR_UNSUPPORTED before anything is launched.  Every GPU that loads the
// library carries the array (about 1.5 MB) until the process exits.  All
// calls on a device share it: calls whose kernels overlap on that device
// (different streams without ordering) race and corrupt each other, so
// order them on one stream.  The valid-row counters start from zero on every
// call (cleared with cudaMemsetAsync, which allocates nothing); the other
// scratch is fully rewritten by each call.
//
// The first call in each CUDA context looks up the array's device address
// with cudaGetSymbolAddress while that context's device is current (a
// host-side lookup, cached per context); make that first call before any
// stream capture.  The cache is keyed by the driver context, so a device
// reset (a new primary context) triggers a fresh lookup instead of reusing a
// stale address.
// ---------------------------------------------------------------------------
namespace {
constexpr int64_t kNoAllocMaxRows = 262144;
constexpr int kNoAllocMaxBatch = 65536;
constexpr int kNoAllocMaxParts = 1024;
constexpr size_t kNoAllocScratchBytes =
    (size_t)kNoAllocMaxRows * sizeof(float) + (size_t)kNoAllocMaxBatch * sizeof(int) +
    (size_t)kNoAllocMaxParts * 2 * sizeof(float) + (size_t)kNoAllocMaxBatch * sizeof(float);
static __device__ __align__(256) unsigned char g_select_scratch[kNoAllocScratchBytes];

std::mutex g_scratch_mu;
std::map<void*, void*> g_scratch_addr;  // driver context -> address of g_select_scratch in it

// The current driver context (CUcontext), through the runtime's driver entry
// point so the library needs no link-time libcuda.
void* current_context() {
  using GetCtx = int (*)(void**);
  static GetCtx fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<GetCtx>(nullptr);
    return reinterpret_cast<GetCtx>(p);
  }();
  void* ctx = nullptr;
  if (!fn || fn(&ctx) != 0) return nullptr;
  return ctx;
}

// Device address of g_select_scratch in the current context (looked up once
// per context).
int select_scratch_address(void** out) {
  void* ctx = current_context();
  if (!ctx) {
    // no context is current yet: the symbol lookup initialises the current
    // device's primary context (and allocates nothing)
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_select_scratch) != cudaSuccess) return MN_ERR_LAUNCH;
    ctx = current_context();
    if (!ctx) return MN_ERR_LAUNCH;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  auto it = g_scratch_addr.find(ctx);
  if (it == g_scratch_addr.end()) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_select_scratch) != cudaSuccess || p == nullptr) return MN_ERR_LAUNCH;
    it = g_scratch_addr.emplace(ctx, p).first;
  }
  *out = it->second;
  return MN_OK;
}
}  // namespace

extern "C" int mn_dtem_select_noalloc(int batch, int num_donors, int k_slots, const float* scores,
                                      const uint8_t* allowed, int k, float tau1, float tau2, float* assignment,
                                      int* status, void* stream) {
  if (batch <= 0 || num_donors <= 0 || k_slots <= 0 || !scores || !allowed || !assignment) return MN_ERR_ARG;
  if (num_donors > 4096) return MN_ERR_UNSUPPORTED;
  const int64_t rows = (int64_t)batch * num_donors;
  if (rows > kNoAllocMaxRows || batch > kNoAllocMaxBatch) return MN_ERR_UNSUPPORTED;
  const int parts = thre_topk_parts(rows);
  if (parts > kNoAllocMaxParts) return MN_ERR_UNSUPPORTED;
  void* scratch = nullptr;
  const int rc = select_scratch_address(&scratch);
  if (rc != MN_OK) return rc;
  cudaGetLastError();
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  float* energy = static_cast<float*>(scratch);
  int* counts = reinterpret_cast<int*>(energy + rows);
  float* partials = reinterpret_cast<float*>(counts + batch);
  float* lam = partials + 2 * parts;
  const int np = next_pow2(num_donors);
  const size_t smem = row_scratch_bytes(np) + (size_t)num_donors * sizeof(float);
  if (k_slots > 160) return MN_ERR_UNSUPPORTED;  // the row kernel stages 256 rows of K slots
  if (!ensure_smem(select_lambda_kernel, smem) || !ensure_smem(select_rows_kernel, (size_t)256 * k_slots * 5))
    return MN_ERR_LAUNCH;
  cudaMemsetAsync(counts, 0, (size_t)batch * sizeof(int), st);
  select_energy_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(scores, allowed, (int)rows, k_slots, tau1,
                                                                   energy, counts, num_donors);
  minmax_partials_kernel<<<parts, 256, 0, st>>>(energy, rows, partials);
  launch_select(batch, num_donors, k_slots, scores, allowed, k, tau1, tau2, energy, counts, partials, parts, lam, smem,
                assignment, status, st);
  return launch_status();
}
