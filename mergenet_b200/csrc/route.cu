// Fused DTEM spatial routing for the canonical eval grouping
// (alternating_per_layer_fast) on sm_100a.
//
// The reference (opentome/timm/dtem.py:1687-2223, driven six times by
// LocalEncoder.forward, opentome/models/mergenet/model.py:574-590, then the
// carrier block model.py:1157-1183) runs ~60 ATen/Triton launches per layer
// and rewrites the full [B,T,C] token tensor six times.  Here the work is
// split by what it depends on:
//
//   route_score    (layer, image, band)  metrics -> compact scores + row energy
//   route_select   (layer, image)        global ThreTopK range -> assignment
//   route_mass     (image)               6-layer mass / centre chain + carriers
//   route_transport(image, channel tile) 6-layer feature transport in shared
//                                        memory + carrier gather
//
// Assignments depend only on metrics (never on tokens or masses), so all
// layers are scored and selected in parallel; only masses, centres and
// features chain through the layers, and features are read once from HBM and
// written once (the carriers).
#include <algorithm>
#include <cstdio>

#include "common.cuh"
#include "thretopk.cuh"

namespace mn {

struct RouteWs {
  float* assign;     // [L][B][half][kc]   scores, then assignment
  float* energy;     // [L][B][half]
  float* asum;       // [L][B][half]       row sums of the assignment
  float* partials;   // [L][B][bands][2]   per-CTA min / max of the energy
  float* wa_old;     // [L][B][half]
  float* wb_old;     // [L][B][half]
  float* wb_safe;    // [L][B][half]
  float* cf;         // [L][B][half][16]  stencil form: [alpha, c_0 .. c_11, 0 ..]
  int32_t* carrier_tok;  // [B][k]      token index of each carrier, in order
};

constexpr int kStencilSlots = 16;
constexpr int kMaxKin = 12;  // receiver in-degree handled with all loads in flight (radius 3)

__host__ inline size_t route_ws_floats(int L, int B, int half, int kc, int bands) {
  return (size_t)L * B * half * kc + (size_t)L * B * half * 5 + (size_t)L * B * bands * 2 +
         (size_t)L * B * half * kStencilSlots;
}

// Table views for layer parity q.
struct ParityTables {
  const int32_t* slot_k;
  const int32_t* slot_rx;
  const int32_t* rx_in;
  const int32_t* rx_off;
};
__host__ __device__ inline ParityTables parity_tables(const int32_t* t, int half, int kc, int kin, int q) {
  const int32_t* base = t + (int64_t)q * ((int64_t)half * kc * 2 + (int64_t)half * kin * 2);
  ParityTables p;
  p.slot_k = base;
  p.slot_rx = base + (int64_t)half * kc;
  p.rx_in = base + (int64_t)half * kc * 2;
  p.rx_off = p.rx_in + (int64_t)half * kin;
  return p;
}

struct KBudget {
  int v[64];  // per-layer merge budget r (passed by value)
};

struct Banding {
  int bands;     // CTAs per (image, layer)
  int rows;      // grid rows per band
  int radius_rows;
  int cap;       // receivers the shared-memory tile holds
};

// ---------------------------------------------------------------------------
// route_score: one CTA per (band, image, layer).  Receivers the band's donors
// can reach are normalised into shared memory (fp32, metric / max(|m|,1e-6)
// as dtem.py:1689-1691); each warp then scores one donor at a time against
// its legal receivers (dtem.py:361-433 restricted to the compact slots) and
// folds the masked logsumexp energy (dtem.py:1557-1567).
// ---------------------------------------------------------------------------
template <int MDT>
__global__ void __launch_bounds__(512) route_score_kernel(
    const typename Elem<MDT>::T* __restrict__ metrics, const int32_t* __restrict__ table,
    int B, int T, int Cm, int grid_w, int half, int kc, int kin, Banding band, float tau1,
    RouteWs ws, int* status) {
  using ET = typename Elem<MDT>::T;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  float* recv = reinterpret_cast<float*>(smem_raw);  // [cap][Cm]
  __shared__ float red[64];

  const int l = blockIdx.y;
  const int b = blockIdx.x / band.bands;
  const int bi = blockIdx.x % band.bands;
  const int q = l & 1;
  const int dp = q ? 0 : 1, rp = 1 - dp;
  const ParityTables pt = parity_tables(table, half, kc, kin, q);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const int grid_h = (2 * half) / grid_w;

  // donor / receiver local ranges of this band
  const int r0 = bi * band.rows, r1 = min(grid_h, r0 + band.rows);
  const int p_lo = r0 * grid_w, p_hi = r1 * grid_w;                  // donor patches
  const int d_lo = (p_lo - dp + 1) >> 1, d_hi = (p_hi - dp + 1) >> 1;  // ceil((p - dp)/2)
  const int rr0 = max(0, r0 - band.radius_rows), rr1 = min(grid_h, r1 + band.radius_rows);
  const int s_lo = (rr0 * grid_w - rp + 1) >> 1, s_hi = (rr1 * grid_w - rp + 1) >> 1;

  const ET* mbase = metrics + ((int64_t)l * B + b) * (int64_t)T * Cm;
  const int per = (Cm + 31) >> 5;  // <= 4

  // normalised receivers -> shared memory
  for (int s = s_lo + warp; s < s_hi; s += nwarps) {
    const ET* row = mbase + (int64_t)(1 + 2 * s + rp) * Cm;
    float v[4];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      int c = lane + 32 * j;
      v[j] = (j < per && c < Cm) ? to_f32(row[c]) : 0.f;
      ss = fmaf(v[j], v[j], ss);
    }
    ss = warp_sum(ss);
    float nrm = fmaxf(sqrtf(ss), 1e-6f);
    float* dst = recv + (int64_t)(s - s_lo) * Cm;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      int c = lane + 32 * j;
      if (j < per && c < Cm) dst[c] = v[j] / nrm;
    }
  }
  __syncthreads();

  float emin = INFINITY, emax = -INFINITY;
  const int64_t lb = (int64_t)l * B + b;
  float* sc_out = ws.assign + lb * half * kc;
  float* e_out = ws.energy + lb * half;
  for (int d = d_lo + warp; d < d_hi; d += nwarps) {
    const ET* row = mbase + (int64_t)(1 + 2 * d + dp) * Cm;
    float a[4];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      int c = lane + 32 * j;
      a[j] = (j < per && c < Cm) ? to_f32(row[c]) : 0.f;
      ss = fmaf(a[j], a[j], ss);
    }
    ss = warp_sum(ss);
    float nrm = fmaxf(sqrtf(ss), 1e-6f);
#pragma unroll
    for (int j = 0; j < 4; ++j) a[j] = a[j] / nrm;
    float mine = -INFINITY;
    const int32_t* srx = pt.slot_rx + (int64_t)d * kc;
    for (int c = 0; c < kc; ++c) {
      int s = srx[c];
      if (s < 0) break;
      if (s < s_lo || s >= s_hi) {  // outside the staged band: a table/banding bug
        if (lane == 0 && status) atomicOr(status, MN_STATUS_TOO_MANY_EDGES);
        continue;
      }
      const float* rv = recv + (int64_t)(s - s_lo) * Cm;
      float acc = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        int cc = lane + 32 * j;
        if (j < per && cc < Cm) acc = fmaf(a[j], rv[cc], acc);
      }
      acc = warp_sum(acc);
      if (lane == c) mine = acc / tau1;
    }
    float m = warp_max(mine);
    float e = 0.f;
    if (m != -INFINITY) {
      float ex = (mine != -INFINITY) ? expf(mine - m) : 0.f;
      float sum = warp_sum(ex);
      e = expf(logf(sum) + m);
    }
    if (lane < kc) sc_out[(int64_t)d * kc + lane] = mine;
    if (lane == 0) e_out[d] = e;
    emin = fminf(emin, e);
    emax = fmaxf(emax, e);
  }
  block_minmax(emin, emax, red);
  if (threadIdx.x == 0) {
    float* p = ws.partials + (lb * band.bands + bi) * 2;
    p[0] = emin;
    p[1] = emax;
  }
}


constexpr int kMaxKc = 16;

// ---------------------------------------------------------------------------
// route_score_lane: the same scores with one thread per donor.  The band's
// receivers are normalised once into shared memory (fp32 rows of CM + 4
// floats, so the rows of consecutive receivers start 16 bytes apart modulo
// 128 and a warp's 16-byte reads spread over all banks); each thread holds
// its donor's normalised row in registers and walks its compact slots, so a
// (donor, slot) edge costs CM / 4 vector loads and CM FMAs with no shuffle.
// ---------------------------------------------------------------------------
template <int CM>
__device__ __forceinline__ void load_metric_row_f32(const float* row, float* v) {
#pragma unroll
  for (int w = 0; w < CM / 4; ++w) {
    const float4 u = __ldg(reinterpret_cast<const float4*>(row) + w);
    v[4 * w] = u.x; v[4 * w + 1] = u.y; v[4 * w + 2] = u.z; v[4 * w + 3] = u.w;
  }
}
template <int CM, typename ET>
__device__ __forceinline__ void load_metric_row(const ET* row, float* v) {
  if constexpr (std::is_same<ET, float>::value) {
    load_metric_row_f32<CM>(row, v);
  } else {
#pragma unroll
    for (int w = 0; w < CM / 8; ++w) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(row) + w);
      const ET* e = reinterpret_cast<const ET*>(&u);
#pragma unroll
      for (int i = 0; i < 8; ++i) v[8 * w + i] = to_f32(e[i]);
    }
  }
}
// metric / max(|metric|, 1e-6) (dtem.py:1689-1691)
template <int CM>
__device__ __forceinline__ void normalise_row(float* v) {
  float s4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int i = 0; i < CM; ++i) s4[i & 3] = fmaf(v[i], v[i], s4[i & 3]);
  const float nr = fmaxf(sqrtf((s4[0] + s4[1]) + (s4[2] + s4[3])), 1e-6f);
#pragma unroll
  for (int i = 0; i < CM; ++i) v[i] = v[i] / nr;
}

constexpr int kLaneScoreThreads = 256;

template <int MDT, int CM>
__global__ void __launch_bounds__(kLaneScoreThreads, 2) route_score_lane_kernel(
    const typename Elem<MDT>::T* __restrict__ metrics, const int32_t* __restrict__ table, int B, int T, int grid_w,
    int half, int kc, int kin, Banding band, float tau1, RouteWs ws, int* status) {
  using ET = typename Elem<MDT>::T;
  constexpr int RS = CM + 4;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ float red[64];
  float* nrm = reinterpret_cast<float*>(smem_raw);  // [s_hi - s_lo][RS]
  const int l = blockIdx.y;
  const int b = blockIdx.x / band.bands;
  const int bi = blockIdx.x % band.bands;
  const int q = l & 1;
  const int dp = q ? 0 : 1, rp = 1 - dp;
  const ParityTables pt = parity_tables(table, half, kc, kin, q);
  const int grid_h = (2 * half) / grid_w;
  const int r0 = bi * band.rows, r1 = min(grid_h, r0 + band.rows);
  const int d_lo = (r0 * grid_w - dp + 1) >> 1, d_hi = (r1 * grid_w - dp + 1) >> 1;
  const int rr0 = max(0, r0 - band.radius_rows), rr1 = min(grid_h, r1 + band.radius_rows);
  const int s_lo = (rr0 * grid_w - rp + 1) >> 1, s_hi = (rr1 * grid_w - rp + 1) >> 1;
  const ET* mbase = metrics + ((int64_t)l * B + b) * (int64_t)T * CM;

  for (int s = s_lo + threadIdx.x; s < s_hi; s += blockDim.x) {
    float v[CM];
    load_metric_row<CM>(mbase + (int64_t)(1 + 2 * s + rp) * CM, v);
    normalise_row<CM>(v);
    float4* dst = reinterpret_cast<float4*>(nrm + (int64_t)(s - s_lo) * RS);
#pragma unroll
    for (int w = 0; w < CM / 4; ++w) dst[w] = make_float4(v[4 * w], v[4 * w + 1], v[4 * w + 2], v[4 * w + 3]);
  }
  __syncthreads();

  float emin = INFINITY, emax = -INFINITY;
  const int64_t lb = (int64_t)l * B + b;
  float* sc_out = ws.assign + lb * half * kc;
  float* e_out = ws.energy + lb * half;
  const bool unit_tau = tau1 == 1.0f;
  for (int d = d_lo + threadIdx.x; d < d_hi; d += blockDim.x) {
    float a[CM];
    load_metric_row<CM>(mbase + (int64_t)(1 + 2 * d + dp) * CM, a);
    normalise_row<CM>(a);
    float2 a2[CM / 2];
#pragma unroll
    for (int i = 0; i < CM / 2; ++i) a2[i] = make_float2(a[2 * i], a[2 * i + 1]);
    const int32_t* srx = pt.slot_rx + (int64_t)d * kc;
    float sc[kMaxKc];
#pragma unroll
    for (int c = 0; c < kMaxKc; ++c) {
      sc[c] = -INFINITY;
      if (c >= kc) continue;
      const int sidx = __ldg(srx + c);
      if (sidx < 0) continue;
      if (sidx < s_lo || sidx >= s_hi) {  // outside the band's receivers: a table error
        if (status) atomicOr(status, MN_STATUS_TOO_MANY_EDGES);
        continue;
      }
      const float4* rv = reinterpret_cast<const float4*>(nrm + (int64_t)(sidx - s_lo) * RS);
      // four accumulators over channels i mod 4, two per fp32x2 FMA (each
      // lane bitwise the scalar FMA)
      float2 acc01 = make_float2(0.f, 0.f), acc23 = make_float2(0.f, 0.f);
#pragma unroll
      for (int w = 0; w < CM / 4; ++w) {
        const float4 r4 = rv[w];
        acc01 = ffma2(a2[2 * w], make_float2(r4.x, r4.y), acc01);
        acc23 = ffma2(a2[2 * w + 1], make_float2(r4.z, r4.w), acc23);
      }
      const float acc = (acc01.x + acc01.y) + (acc23.x + acc23.y);
      // logits = scores / tau1 (dtem.py:1557); exact without a division at tau1 == 1
      sc[c] = unit_tau ? acc : acc / tau1;
    }
    float m = -INFINITY;
#pragma unroll
    for (int c = 0; c < kMaxKc; ++c) m = fmaxf(m, sc[c]);
    float e = 0.f;
    if (m != -INFINITY) {
      float sum = 0.f;
#pragma unroll
      for (int c = 0; c < kMaxKc; ++c)
        if (sc[c] != -INFINITY) sum += expf(sc[c] - m);
      e = expf(logf(sum) + m);
    }
    float* dst = sc_out + (int64_t)d * kc;
    if (kc == 12) {  // the radius-3 compact width: three aligned 16-byte stores
      float4* d4 = reinterpret_cast<float4*>(dst);
      d4[0] = make_float4(sc[0], sc[1], sc[2], sc[3]);
      d4[1] = make_float4(sc[4], sc[5], sc[6], sc[7]);
      d4[2] = make_float4(sc[8], sc[9], sc[10], sc[11]);
    } else {
#pragma unroll
      for (int c = 0; c < kMaxKc; ++c)
        if (c < kc) dst[c] = sc[c];
    }
    e_out[d] = e;
    emin = fminf(emin, e);
    emax = fmaxf(emax, e);
  }
  block_minmax(emin, emax, red);
  if (threadIdx.x == 0) {
    float* p = ws.partials + (lb * band.bands + bi) * 2;
    p[0] = emin;
    p[1] = emax;
  }
}

// ---------------------------------------------------------------------------
// route_select: one CTA per (image, layer), kSelectThreads threads.  Global
// ThreTopK range over the whole batch for this layer (thetopk.py:12-13), the
// per-row threshold (block-wide, keys sorted in registers), then the masked
// softmax x row k-hot and the clamp-normalise of every donor row
// (dtem.py:1568-1579), with the row's slots in registers.
// ---------------------------------------------------------------------------
constexpr int kSelectThreads = 256;

__global__ void __launch_bounds__(kSelectThreads) route_select_kernel(
    const int32_t* __restrict__ table, int B, int half, int kc, int kin, int bands,
    KBudget kb, float tau2, RouteWs ws, int* status) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int np = next_pow2(half);
  RowScratch rs = carve_row_scratch(smem_raw, np);
  float* xrow = reinterpret_cast<float*>(smem_raw + row_scratch_bytes(np));  // [half] scaled energies
  __shared__ float red[64];

  const int b = blockIdx.x, l = blockIdx.y, q = l & 1;
  const int64_t lb = (int64_t)l * B + b;
  const ParityTables pt = parity_tables(table, half, kc, kin, q);

  // batch-global range of this layer's energies
  float gmin = INFINITY, gmax = -INFINITY;
  const float* part = ws.partials + (int64_t)l * B * bands * 2;
  for (int i = threadIdx.x; i < B * bands; i += blockDim.x) {
    gmin = fminf(gmin, part[2 * i]);
    gmax = fmaxf(gmax, part[2 * i + 1]);
  }
  block_minmax(gmin, gmax, red);
  const float range = gmax - gmin;
  if (threadIdx.x == 0 && b == 0 && !(range > 0.f && range < INFINITY) && status)
    atomicOr(status, MN_STATUS_DEGENERATE_RANGE);

  const float* e = ws.energy + lb * half;
  for (int d = threadIdx.x; d < half; d += blockDim.x) xrow[d] = e[d] / range * tau2;
  __syncthreads();
  const float lam = thre_topk_lambda(xrow, half, np, kb.v[l], rs);

  float* asg = ws.assign + lb * half * kc;
  float* asum = ws.asum + lb * half;
  for (int d = threadIdx.x; d < half; d += blockDim.x) {
    float* row = asg + (int64_t)d * kc;
    const int32_t* srx = pt.slot_rx + (int64_t)d * kc;
    float sc[kMaxKc];
    int sl[kMaxKc];
#pragma unroll
    for (int c = 0; c < kMaxKc; ++c) {  // every load in flight before any use
      sc[c] = c < kc ? row[c] : -INFINITY;
      sl[c] = c < kc ? __ldg(srx + c) : -1;
    }
    int cnt = 0;  // legal slots come first (the compact table's order)
#pragma unroll
    for (int c = 0; c < kMaxKc; ++c)
      if (cnt == c && sl[c] >= 0) ++cnt;
    if (cnt == 0) {
      asum[d] = 0.f;
      continue;
    }
    float m = -INFINITY;
#pragma unroll
    for (int c = 0; c < kMaxKc; ++c)
      if (c < cnt) m = fmaxf(m, sc[c]);
    const float y = thre_topk_map(xrow[d], lam);  // row k-hot (valid row)
    float sum = 0.f;
#pragma unroll
    for (int c = 0; c < kMaxKc; ++c)
      if (c < cnt) sum += expf(sc[c] - m);
    const float inv = 1.0f / sum;
    float ks = 0.f;
#pragma unroll
    for (int c = 0; c < kMaxKc; ++c) {
      if (c < cnt) {
        sc[c] = (expf(sc[c] - m) * inv) * y;  // khot
        ks += sc[c];
      }
    }
    const float tmp = fmaxf(ks - 1.0f, 0.0f) + 1.0f;
    float as = 0.f;
#pragma unroll
    for (int c = 0; c < kMaxKc; ++c) {
      if (c < kc) {
        const float v = c < cnt ? sc[c] / tmp : 0.f;
        row[c] = v;
        as += v;
      }
    }
    asum[d] = as;
  }
}

// ---------------------------------------------------------------------------
// route_mass: one CTA per image, kMassThreads threads.  Mass and
// centre-of-mass chain over the layers (dtem.py:1978-1983, :2016-2025,
// :2027-2044, interleave :2196-2222), then the exact top-k by mass and the
// centre-of-mass ordering (model.py:1167-1171).  A receiver's update reads
// only its own state and its donors' old masses and centres, and a donor's
// only its own mass, so each layer updates the receivers in place, then
// (after a barrier) the donors.  It also writes the coefficients of the
// feature transport.
// ---------------------------------------------------------------------------
constexpr int kMassThreads = 512;

__host__ __device__ inline size_t align16(size_t v) { return (v + 15) & ~size_t(15); }
__host__ __device__ inline size_t mass_smem_bytes(int T, int k) {
  const int np = next_pow2(T - 1), nk = next_pow2(k);
  const int nx = np > kMassThreads ? np : kMassThreads;
  return align16((size_t)2 * T * 4) + (size_t)(np + nk) * 8 + (size_t)2 * nx * 8;
}

// Sort the n keys key_of(0 .. n-1) (n a power of two <= R * bd) into out[0 .. n).
template <int R, typename KeyOf>
__device__ __forceinline__ void sort_carrier_keys(int n, int bd, KeyOf key_of, unsigned long long* out,
                                                  unsigned long long* xbuf) {
  unsigned long long kv[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int idx = threadIdx.x + r * bd;
    kv[r] = idx < n ? key_of(idx) : ~0ull;
  }
  bitonic_sort_regs<R>(kv, xbuf, n);
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int idx = threadIdx.x + r * bd;
    if (idx < n) out[idx] = kv[r];
  }
}
template <typename KeyOf>
__device__ __forceinline__ void sort_carrier_keys_any(int n, int bd, KeyOf key_of, unsigned long long* out,
                                                      unsigned long long* xbuf) {
  const int r = n > bd ? n / bd : 1;
  if (r == 1) sort_carrier_keys<1>(n, bd, key_of, out, xbuf);
  else if (r == 2) sort_carrier_keys<2>(n, bd, key_of, out, xbuf);
  else if (r == 4) sort_carrier_keys<4>(n, bd, key_of, out, xbuf);
  else sort_carrier_keys<8>(n, bd, key_of, out, xbuf);
}

__global__ void __launch_bounds__(kMassThreads, 2) route_mass_kernel(
    const int32_t* __restrict__ table, int B, int T, int half, int kc, int kin, int L, int k,
    int write_stencil, RouteWs ws, float* __restrict__ size_out, float* __restrict__ center_out,
    float* __restrict__ topk_size, int64_t* __restrict__ topk_idx) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  float* size = reinterpret_cast<float*>(smem_raw);  // [T]
  float* center = size + T;                          // [T]
  const int P = T - 1;
  const int np = next_pow2(P), nk = next_pow2(k);
  unsigned long long* keys = reinterpret_cast<unsigned long long*>(smem_raw + align16((size_t)2 * T * 4));
  unsigned long long* keys2 = keys + np;
  unsigned long long* xbuf = keys2 + nk;  // exchange buffers of the sorts
  const int b = blockIdx.x;
  const float eps = 1.1920928955078125e-07f;  // torch.finfo(float32).eps

  for (int t = threadIdx.x; t < T; t += blockDim.x) {
    size[t] = 1.0f;
    center[t] = (float)t;
  }
  __syncthreads();
  for (int l = 0; l < L; ++l) {
    const int q = l & 1, dp = q ? 0 : 1, rp = 1 - dp;
    const ParityTables pt = parity_tables(table, half, kc, kin, q);
    const int64_t lb = (int64_t)l * B + b;
    const float* asg = ws.assign + lb * half * kc;
    const float* asum = ws.asum + lb * half;
    // receivers, in place (they read donors' old masses and centres only)
    for (int i = threadIdx.x; i < half; i += blockDim.x) {
      const int tb = 1 + 2 * i + rp;
      const float wb = size[tb], cb = center[tb];
      float contrib = 0.f, ccontrib = 0.f;
      const int32_t* in = pt.rx_in + (int64_t)i * kin;
      const int32_t* off = pt.rx_off + (int64_t)i * kin;
      // the in-edges in the reference's sequential scatter order; with up to
      // kMaxKin of them every load is in flight before the sums
      const bool fast_in = kin <= kMaxKin;
      int ev[kMaxKin], ov[kMaxKin];
      float wv[kMaxKin];
      if (fast_in) {
#pragma unroll
        for (int j = 0; j < kMaxKin; ++j) {
          ev[j] = j < kin ? __ldg(in + j) : -1;
          ov[j] = (write_stencil && j < kin) ? __ldg(off + j) : -1;
        }
#pragma unroll
        for (int j = 0; j < kMaxKin; ++j) wv[j] = ev[j] >= 0 ? __ldg(asg + ev[j]) : 0.f;
#pragma unroll
        for (int j = 0; j < kMaxKin; ++j) {
          if (ev[j] < 0) break;
          const int ta = 1 + 2 * (ev[j] / kc) + dp;
          const float wa = size[ta];
          contrib = __fadd_rn(contrib, __fmul_rn(wv[j], wa));
          ccontrib = __fadd_rn(ccontrib, __fmul_rn(wv[j], __fmul_rn(wa, center[ta])));
        }
      } else {
        for (int j = 0; j < kin; ++j) {
          const int e = __ldg(in + j);
          if (e < 0) break;
          const float w = __ldg(asg + e);
          const int ta = 1 + 2 * (e / kc) + dp;
          const float wa = size[ta];
          contrib = __fadd_rn(contrib, __fmul_rn(w, wa));
          ccontrib = __fadd_rn(ccontrib, __fmul_rn(w, __fmul_rn(wa, center[ta])));
        }
      }
      const float wbn = __fadd_rn(wb, contrib);
      const float wsafe = fmaxf(wbn, eps);
      if (write_stencil) {
        // x_s <- alpha * x_s + sum_j c_j * x_dj, the same update scaled by
        // 1 / wb_safe once per coefficient instead of once per channel.
        // Chunk-major: slot u of receiver i at ((lb * 4 + u / 4) * half + i) * 4 + u % 4;
        // absent slots are zero (written first, then the present edges).
        float* cf = ws.cf + (lb * 4 * half + i) * 4;
        auto cf_slot = [&](int u) -> float* { return cf + (int64_t)(u >> 2) * half * 4 + (u & 3); };
#pragma unroll
        for (int w = 0; w < kStencilSlots / 4; ++w)
          *reinterpret_cast<float4*>(cf + (int64_t)w * half * 4) = make_float4(0.f, 0.f, 0.f, 0.f);
        *cf_slot(0) = wb / wsafe;
        if (fast_in) {
#pragma unroll
          for (int j = 0; j < kMaxKin; ++j) {
            if (ev[j] < 0) break;
            const float v = (wv[j] * size[1 + 2 * (ev[j] / kc) + dp]) / wsafe;
            if (ov[j] >= 0 && ov[j] + 1 < kStencilSlots) *cf_slot(ov[j] + 1) = v;
          }
        } else {
          for (int j = 0; j < kin; ++j) {
            const int e = __ldg(in + j);
            if (e < 0) break;
            const int o = __ldg(off + j);
            const float v = (__ldg(asg + e) * size[1 + 2 * (e / kc) + dp]) / wsafe;
            if (o >= 0 && o + 1 < kStencilSlots) *cf_slot(o + 1) = v;
          }
        }
      } else {
        // the table-driven transport reads the old masses of both sides
        ws.wb_old[lb * half + i] = wb;
        ws.wb_safe[lb * half + i] = wsafe;
        ws.wa_old[lb * half + i] = size[1 + 2 * i + dp];  // donor i, not yet updated
      }
      size[tb] = wbn;
      center[tb] = __fdiv_rn(__fadd_rn(__fmul_rn(wb, cb), ccontrib), wsafe);
    }
    __syncthreads();
    // donors (their own old mass and assignment row sum only)
    for (int i = threadIdx.x; i < half; i += blockDim.x) {
      const int ta = 1 + 2 * i + dp;
      const float tmp = __fsub_rn(1.0f, __ldg(asum + i));
      size[ta] = __fmul_rn(size[ta], fminf(fmaxf(tmp, 0.f), 1.f));
    }
    if (threadIdx.x == 0) center[0] = 0.f;  // CLS centre after the first layer
    __syncthreads();
  }
  for (int t = threadIdx.x; t < T; t += blockDim.x) {
    size_out[(int64_t)b * T + t] = size[t];
    center_out[(int64_t)b * T + t] = center[t];
  }
  // exact top-k by (mass desc, patch asc): key = (~bits(mass) << 32) | patch
  auto mass_key = [&](int i) -> unsigned long long {
    if (i >= P) return ~0ull;
    const unsigned int bits = __float_as_uint(size[1 + i]);
    return ((unsigned long long)(~bits) << 32) | (unsigned int)i;
  };
  const int bd = blockDim.x;
  sort_carrier_keys_any(np, bd, mass_key, keys, xbuf);
  __syncthreads();
  // re-key the k winners by (centre asc, patch asc); centres are >= 0
  auto centre_key = [&](int i) -> unsigned long long {
    if (i >= k) return ~0ull;
    const unsigned int p = (unsigned int)(keys[i] & 0xffffffffu);
    return ((unsigned long long)__float_as_uint(center[1 + p]) << 32) | p;
  };
  sort_carrier_keys_any(nk, bd, centre_key, keys2, xbuf);
  __syncthreads();
  for (int i = threadIdx.x; i < k; i += blockDim.x) {
    unsigned int p = (unsigned int)(keys2[i] & 0xffffffffu);
    topk_idx[(int64_t)b * k + i] = p;
    ws.carrier_tok[(int64_t)b * k + i] = (int)p + 1;
    topk_size[(int64_t)b * (k + 1) + 1 + i] = size[1 + p];
  }
  if (threadIdx.x == 0) topk_size[(int64_t)b * (k + 1)] = size[0];
}

// Stage x[b][0..T)[c0 .. c0+CT) into the fp32 shared tile [T][CT].  Full,
// aligned tiles issue every load before the first use: cp.async for fp32,
// 16-byte vector loads batched 8 deep for fp16 / bf16.
template <typename XT, int CT>
__device__ __forceinline__ void load_token_tile(float* tile, const XT* __restrict__ xb, int T, int C, int c0) {
  const bool vec = (c0 + CT <= C) && (C % 8 == 0) && ((reinterpret_cast<uintptr_t>(xb) & 15) == 0);
  if (!vec) {
    for (int i = threadIdx.x; i < T * CT; i += blockDim.x) {
      const int t = i / CT, c = i % CT;
      tile[i] = (c0 + c < C) ? to_f32(xb[(int64_t)t * C + c0 + c]) : 0.f;
    }
    return;
  }
  if (sizeof(XT) == 4) {
    constexpr int VPR = CT / 4;  // 16-byte vectors per row
    const uint32_t sbase = static_cast<uint32_t>(__cvta_generic_to_shared(tile));
    for (int i = threadIdx.x; i < T * VPR; i += blockDim.x) {
      const int t = i / VPR, v = i % VPR;
      const void* src = xb + (int64_t)t * C + c0 + 4 * v;
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(sbase + (uint32_t)(t * CT + 4 * v) * 4u),
                   "l"(src) : "memory");
    }
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
    return;
  }
  constexpr int VPR = CT / 8;  // 16-byte vectors (8 halves) per row
  const int nvec = T * VPR;
  for (int i0 = threadIdx.x; i0 < nvec; i0 += 8 * blockDim.x) {
    uint4 buf[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = i0 + u * blockDim.x;
      if (i < nvec) buf[u] = *reinterpret_cast<const uint4*>(xb + (int64_t)(i / VPR) * C + c0 + 8 * (i % VPR));
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = i0 + u * blockDim.x;
      if (i >= nvec) break;
      const XT* e = reinterpret_cast<const XT*>(&buf[u]);
      float* dst = tile + (i / VPR) * CT + 8 * (i % VPR);
      *reinterpret_cast<float4*>(dst) = make_float4(to_f32(e[0]), to_f32(e[1]), to_f32(e[2]), to_f32(e[3]));
      *reinterpret_cast<float4*>(dst + 4) = make_float4(to_f32(e[4]), to_f32(e[5]), to_f32(e[6]), to_f32(e[7]));
    }
  }
}

// Gather the CLS row and the k carriers out of the shared tile.
template <typename XT, int CT>
__device__ __forceinline__ void store_carriers(XT* __restrict__ out, const float* tile, const int32_t* ctok, int k,
                                               int C, int c0) {
  if (c0 + CT <= C && C % 4 == 0 && ((reinterpret_cast<uintptr_t>(out) & 15) == 0)) {
    constexpr int VPR = CT / 4;
    for (int i = threadIdx.x; i < (k + 1) * VPR; i += blockDim.x) {
      const int r = i / VPR, v = i % VPR;
      const int t = (r == 0) ? 0 : ctok[r - 1];
      const float4 val = *reinterpret_cast<const float4*>(tile + t * CT + 4 * v);
      XT* dst = out + (int64_t)r * C + c0 + 4 * v;
      if (sizeof(XT) == 4) {
        *reinterpret_cast<float4*>(dst) = val;
      } else {
        XT h[4] = {from_f32<XT>(val.x), from_f32<XT>(val.y), from_f32<XT>(val.z), from_f32<XT>(val.w)};
        *reinterpret_cast<uint2*>(dst) = *reinterpret_cast<const uint2*>(h);
      }
    }
    return;
  }
  for (int i = threadIdx.x; i < (k + 1) * CT; i += blockDim.x) {
    const int r = i / CT, cc = i % CT;
    if (c0 + cc >= C) continue;
    const int t = (r == 0) ? 0 : ctok[r - 1];
    out[(int64_t)r * C + c0 + cc] = from_f32<XT>(tile[t * CT + cc]);
  }
}

// ---------------------------------------------------------------------------
// route_transport: one CTA per (image, CT-channel tile).  The token tile
// [T][CT] lives in shared memory in fp32; each layer updates the receivers in
// place (donor features are unchanged by a layer, dtem.py:1973-2025):
//   x_s <- (wb_old[s] * x_s + sum_edges assign * (wa_old[d] * x_d)) / wb_safe[s]
// accumulated in the reference's edge order, then the carriers are gathered.
// ---------------------------------------------------------------------------
template <typename XT, int CT>
__global__ void __launch_bounds__(256) route_transport_kernel(
    const XT* __restrict__ x, const int32_t* __restrict__ table, int B, int T, int C, int half,
    int kc, int kin, int L, int k, RouteWs ws, XT* __restrict__ topk_x) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  float* tile = reinterpret_cast<float*>(smem_raw);  // [T][CT]
  const int b = blockIdx.x;
  const int c0 = blockIdx.y * CT;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  constexpr int RPW = 32 / CT;  // receivers per warp pass
  const int sub = lane / CT, ch = lane % CT;
  const bool ch_ok = (c0 + ch) < C;

  const XT* xb = x + (int64_t)b * T * C;
  load_token_tile<XT, CT>(tile, xb, T, C, c0);
  __syncthreads();
  for (int l = 0; l < L; ++l) {
    const int q = l & 1, dp = q ? 0 : 1, rp = 1 - dp;
    const ParityTables pt = parity_tables(table, half, kc, kin, q);
    const int64_t lb = (int64_t)l * B + b;
    const float* asg = ws.assign + lb * half * kc;
    const float* wa_old = ws.wa_old + lb * half;
    const float* wb_old = ws.wb_old + lb * half;
    const float* wb_safe = ws.wb_safe + lb * half;
    for (int s0 = warp * RPW; s0 < half; s0 += nwarps * RPW) {
      const int s = s0 + sub;
      if (s < half) {
        const int32_t* in = pt.rx_in + (int64_t)s * kin;
        float acc = 0.f;
        for (int j = 0; j < kin; ++j) {
          int e = in[j];
          if (e < 0) break;
          int d = e / kc;
          float t = __fmul_rn(wa_old[d], tile[(1 + 2 * d + dp) * CT + ch]);
          acc = __fadd_rn(acc, __fmul_rn(asg[e], t));
        }
        float* xs = tile + (1 + 2 * s + rp) * CT + ch;
        *xs = __fdiv_rn(__fadd_rn(__fmul_rn(wb_old[s], *xs), acc), wb_safe[s]);
      }
    }
    __syncthreads();
  }
  store_carriers<XT, CT>(topk_x + (int64_t)b * (k + 1) * C, tile, ws.carrier_tok + (int64_t)b * k, k, C, c0);
  (void)ch_ok;
}


// ---------------------------------------------------------------------------
// route_transport_stencil: the same per-layer update for even-width grids,
// where receivers fill whole grid columns and a receiver's donors sit at odd
// column offsets dx in {-3,-1,1,3} and |dy| <= DY1 (|dx| = 1) or DY3
// (|dx| = 3).  The coefficients (alpha = wb_old / wb_safe, c = assign *
// wa_old / wb_safe) come from route_mass in stencil order, chunk-major: the
// 16-byte chunk w of receiver s at ((layer * B + b) * 4 + w) * half + s, so
// the chunks a warp reads for consecutive receivers are contiguous.
//
// The kernel is bound by the L1 data pipe (shared-memory wavefronts), so the
// work is shaped for reuse per shared-memory load: a thread owns 4 channels
// of a PAIR of receiver columns c and c + 2 and walks their rows with a
// sliding window over the three donor columns c - 1, c + 1, c + 3.  Every
// window value it loads serves 2 * DY1 + 1 rows, and the middle column serves
// both receivers; column c + 3 also gives c its dx = +3 donors and c - 1
// gives c + 2 its dx = -3 donors, so only c - 3 and c + 5 are extra loads.
// The next row's coefficient lines are prefetched into L1 one row ahead.
// ---------------------------------------------------------------------------
constexpr int kPairThreads = 256;
#ifndef MN_ROUTE_SPLITS
#define MN_ROUTE_SPLITS 10
#endif
#ifndef MN_ROUTE_NARROW_THREADS
#define MN_ROUTE_NARROW_THREADS 512
#endif
constexpr int kPairSplits = MN_ROUTE_SPLITS;
// Launch bound of the stencil: 32-channel tiles run two CTAs per SM; a
// narrower tile (grids whose token tile does not fit twice, e.g. 48 x 48)
// runs one CTA per SM with up to 512 threads, its rows split ten ways
// (48 x 48, B=64: 819 us for the routing call against 952 us with 256
// threads and four splits; 768 or 1024 threads were slower)
#ifndef MN_ROUTE_WIDE_THREADS
#define MN_ROUTE_WIDE_THREADS 256  // one CTA per SM with 448 or 512 threads: 847-852 against 745 us at 28 x 28
#endif
#ifndef MN_ROUTE_WIDE_BLOCKS
#define MN_ROUTE_WIDE_BLOCKS 2
#endif
template <int CT>
struct StencilBound {
  static constexpr int kThreads = CT == 32 ? MN_ROUTE_WIDE_THREADS : MN_ROUTE_NARROW_THREADS;
  static constexpr int kBlocks = CT == 32 ? MN_ROUTE_WIDE_BLOCKS : 1;
};

template <typename XT, int CT, int DY1, int DY3>
__global__ void __launch_bounds__(StencilBound<CT>::kThreads, StencilBound<CT>::kBlocks)
    route_transport_stencil_kernel(
    const XT* __restrict__ x, int B, int T, int C, int grid_h, int grid_w, int half, int L, int k,
    int row_splits, RouteWs ws, XT* __restrict__ topk_x) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  float* tile = reinterpret_cast<float*>(smem_raw);  // [T][CT]
  constexpr int G = CT / 4;                           // float4 channel groups
  constexpr int NW = 2 * DY1 + 1;                     // window rows
  static_assert(DY3 <= DY1, "the dx = 3 donors of one column lie inside the next pair column's window");
  const int b = blockIdx.x;
  const int c0 = blockIdx.y * CT;
  const XT* xb = x + (int64_t)b * T * C;
  load_token_tile<XT, CT>(tile, xb, T, C, c0);
  float* zrow = tile + (int64_t)T * CT;  // one row of zeros after the tile
  for (int i = threadIdx.x; i < CT; i += blockDim.x) zrow[i] = 0.f;
  __syncthreads();
  const int half_w = grid_w >> 1;
  const int npairs = (half_w + 1) >> 1;
  const int g = threadIdx.x % G;
  const int pr = (threadIdx.x / G) % npairs;
  const int rs = threadIdx.x / (G * npairs);
  const bool active = rs < row_splits;
  const int rows_per = (grid_h + row_splits - 1) / row_splits;
  const int r_begin = rs * rows_per, r_end = active ? min(grid_h, r_begin + rows_per) : r_begin;
  const int rstride = grid_w * CT;  // floats between grid rows
  const float* zero4 = zrow + 4 * g;
  const int64_t cf_chunk = (int64_t)half * 4;  // floats between chunks w and w + 1
  // acc (two float2 halves) += w * v
  auto fma4 = [](float w, float4 v, float2& lo, float2& hi) {
    const float2 ww = make_float2(w, w);
    lo = ffma2(ww, make_float2(v.x, v.y), lo);
    hi = ffma2(ww, make_float2(v.z, v.w), hi);
  };
  for (int l = 0; l < L; ++l) {
    const int rp = l & 1;       // receiver patch parity = column parity
    const int ca = 4 * pr + rp;  // the pair's columns ca and cb = ca + 2
    const int cb = ca + 2;
    const bool has_b = cb < grid_w;
    // a column outside the grid reads the zero row (its coefficients are zero)
    auto colp = [&](int c) -> const float* {
      return (c >= 0 && c < grid_w) ? tile + (1 + c) * CT + 4 * g : nullptr;
    };
    const float* w0 = colp(ca - 1);
    const float* w1 = colp(ca + 1);
    const float* w2 = colp(ca + 3);
    const float* e0 = colp(ca - 3);
    const float* e1 = colp(ca + 5);
    auto ldc = [&](const float* col, int r) -> float4 {
      const float* src = (col != nullptr && (unsigned)r < (unsigned)grid_h) ? col + r * rstride : zero4;
      return *reinterpret_cast<const float4*>(src);
    };
    const float* cfl = ws.cf + ((int64_t)l * B + b) * 4 * cf_chunk;
    // coefficients of row r for both receivers (chunk-major, 16 bytes each)
    auto load_cf = [&](int r, float4* qa, float4* qb) {
      const int sa = (r * grid_w + ca) >> 1;  // receiver of column ca; cb's is sa + 1
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        qa[w] = __ldg(reinterpret_cast<const float4*>(cfl + w * cf_chunk + (int64_t)sa * 4));
        qb[w] = has_b ? __ldg(reinterpret_cast<const float4*>(cfl + w * cf_chunk + (int64_t)(sa + 1) * 4))
                      : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    };
    float4 v0[NW], v1[NW], v2[NW];
#pragma unroll
    for (int u = 0; u < NW - 1; ++u) {
      v0[u] = ldc(w0, r_begin - DY1 + u);
      v1[u] = ldc(w1, r_begin - DY1 + u);
      v2[u] = ldc(w2, r_begin - DY1 + u);
    }
    for (int rb = r_begin; rb < r_end; rb += NW) {
#pragma unroll
      for (int ph = 0; ph < NW; ++ph) {
        const int r = rb + ph;
        if (r < r_end) {
          const int sa = (r * grid_w + ca) >> 1;  // receiver of column ca; cb's is sa + 1
          if (r + 1 < r_end && g < 4)  // next row's chunk g of both receivers -> L1
            asm volatile("prefetch.global.L1 [%0];" ::"l"(cfl + g * cf_chunk + (int64_t)(sa + half_w) * 4));
          float4 qa[4], qb[4];
          load_cf(r, qa, qb);
          v0[(ph + NW - 1) % NW] = ldc(w0, r + DY1);
          v1[(ph + NW - 1) % NW] = ldc(w1, r + DY1);
          v2[(ph + NW - 1) % NW] = ldc(w2, r + DY1);
          const float cwa[16] = {qa[0].x, qa[0].y, qa[0].z, qa[0].w, qa[1].x, qa[1].y, qa[1].z, qa[1].w,
                                 qa[2].x, qa[2].y, qa[2].z, qa[2].w, qa[3].x, qa[3].y, qa[3].z, qa[3].w};
          const float cwb[16] = {qb[0].x, qb[0].y, qb[0].z, qb[0].w, qb[1].x, qb[1].y, qb[1].z, qb[1].w,
                                 qb[2].x, qb[2].y, qb[2].z, qb[2].w, qb[3].x, qb[3].y, qb[3].z, qb[3].w};
          float4* own_a = reinterpret_cast<float4*>(tile + (1 + r * grid_w + ca) * CT + 4 * g);
          float4* own_b = reinterpret_cast<float4*>(tile + (1 + r * grid_w + (has_b ? cb : ca)) * CT + 4 * g);
          const float4 xa = *own_a, xbv = *own_b;
          float2 la = make_float2(cwa[0] * xa.x, cwa[0] * xa.y), ha = make_float2(cwa[0] * xa.z, cwa[0] * xa.w);
          float2 lb = make_float2(cwb[0] * xbv.x, cwb[0] * xbv.y), hb = make_float2(cwb[0] * xbv.z, cwb[0] * xbv.w);
          int j = 1;
          // column ca: dx = -3 (extra column), -1 (v0), +1 (v1), +3 (v2 rows |dy| <= DY3)
          // column cb: dx = -3 (v0 rows |dy| <= DY3), -1 (v1), +1 (v2), +3 (extra column)
          if (DY3 >= 0) {
#pragma unroll
            for (int dy = -DY3; dy <= DY3; ++dy) {
              fma4(cwa[j], ldc(e0, r + dy), la, ha);
              fma4(cwb[j], v0[(ph + DY1 + dy) % NW], lb, hb);
              ++j;
            }
          }
#pragma unroll
          for (int u = 0; u < NW; ++u) {
            fma4(cwa[j], v0[(ph + u) % NW], la, ha);
            fma4(cwb[j], v1[(ph + u) % NW], lb, hb);
            ++j;
          }
#pragma unroll
          for (int u = 0; u < NW; ++u) {
            fma4(cwa[j], v1[(ph + u) % NW], la, ha);
            fma4(cwb[j], v2[(ph + u) % NW], lb, hb);
            ++j;
          }
          if (DY3 >= 0) {
#pragma unroll
            for (int dy = -DY3; dy <= DY3; ++dy) {
              fma4(cwa[j], v2[(ph + DY1 + dy) % NW], la, ha);
              fma4(cwb[j], ldc(e1, r + dy), lb, hb);
              ++j;
            }
          }
          *own_a = make_float4(la.x, la.y, ha.x, ha.y);
          if (has_b) *own_b = make_float4(lb.x, lb.y, hb.x, hb.y);
        }
      }
    }
    __syncthreads();
  }
  store_carriers<XT, CT>(topk_x + (int64_t)b * (k + 1) * C, tile, ws.carrier_tok + (int64_t)b * k, k, C, c0);
}

static Banding make_banding(int grid_h, int grid_w, int radius_rows, int Cm) {
  Banding bd;
  bd.radius_rows = radius_rows;
  const int max_smem = 110 * 1024;
  bd.cap = max_smem / (Cm * 4);
  for (int nb = 1; nb <= grid_h; ++nb) {
    const int rows = (grid_h + nb - 1) / nb;
    const int need_rows = (nb == 1) ? grid_h : std::min(grid_h, rows + 2 * radius_rows);
    const int need = (need_rows * grid_w + 1) / 2 + 1;
    if (need <= bd.cap) {
      bd.bands = (grid_h + rows - 1) / rows;
      bd.rows = rows;
      return bd;
    }
  }
  bd.bands = -1;
  bd.rows = 0;
  return bd;
}

}  // namespace mn

using namespace mn;

extern "C" size_t mn_route_workspace_bytes(const mn_route_dims* dims, int batch, int num_layers) {
  if (!dims || batch <= 0 || num_layers <= 0) return 0;
  size_t floats = route_ws_floats(num_layers, batch, dims->half, dims->kc, dims->grid_h);
  return floats * sizeof(float) + (size_t)batch * dims->num_patches * sizeof(int32_t);
}

template <typename XT>
static bool launch_transport(const void* x, const int32_t* table, int B, int T, int C, int half, int kc,
                             int kin, int L, int k, const RouteWs& ws, void* topk_x, int ct,
                             cudaStream_t st) {
  size_t smem = (size_t)T * ct * sizeof(float);
  dim3 grid(B, (C + ct - 1) / ct);
  const XT* xp = static_cast<const XT*>(x);
  XT* op = static_cast<XT*>(topk_x);
  if (ct == 32) {
    if (!ensure_smem(route_transport_kernel<XT, 32>, smem)) return false;
    route_transport_kernel<XT, 32><<<grid, 256, smem, st>>>(xp, table, B, T, C, half, kc, kin, L, k, ws, op);
  } else if (ct == 16) {
    if (!ensure_smem(route_transport_kernel<XT, 16>, smem)) return false;
    route_transport_kernel<XT, 16><<<grid, 256, smem, st>>>(xp, table, B, T, C, half, kc, kin, L, k, ws, op);
  } else {
    if (!ensure_smem(route_transport_kernel<XT, 8>, smem)) return false;
    route_transport_kernel<XT, 8><<<grid, 256, smem, st>>>(xp, table, B, T, C, half, kc, kin, L, k, ws, op);
  }
  return true;
}

// Which compiled stencil fits the geometry: 1 = (DY1 2, DY3 0) radius 3,
// 2 = (1, none) radius in [sqrt 2, sqrt 5), 3 = (0, none); 0 = generic path.
static int stencil_variant(const mn_route_dims* d) {
  // 8 channel groups per receiver-column pair must fit the launch bound
  if (d->grid_w % 2 != 0 || ((d->grid_w / 2 + 1) / 2) * 8 > kPairThreads) return 0;
  if (d->stencil_dy1 == 2 && d->stencil_dy3 == 0) return 1;
  if (d->stencil_dy1 == 1 && d->stencil_dy3 == -1) return 2;
  if (d->stencil_dy1 == 0 && d->stencil_dy3 == -1) return 3;
  return 0;
}

template <typename XT, int CT, int DY1, int DY3>
static bool launch_stencil_ct(const void* x, int B, int T, int C, const mn_route_dims* d, int L, int k,
                              const RouteWs& ws, void* topk_x, cudaStream_t st) {
  const int half_w = d->grid_w / 2;
  const int per_split = (CT / 4) * ((half_w + 1) / 2);  // threads per row split
  int splits = std::max(1, std::min(d->grid_h, StencilBound<CT>::kThreads / per_split));  // <= the launch bound
  splits = std::min(splits, kPairSplits);
  const int threads = ((per_split * splits + 31) / 32) * 32;
  const size_t smem = (size_t)(T + 1) * CT * sizeof(float);  // tile + zero row
  auto kern = route_transport_stencil_kernel<XT, CT, DY1, DY3>;
  if (!ensure_smem(kern, smem)) return false;
  kern<<<dim3(B, (C + CT - 1) / CT), threads, smem, st>>>(static_cast<const XT*>(x), B, T, C, d->grid_h,
                                                            d->grid_w, d->half, L, k, splits, ws,
                                                            static_cast<XT*>(topk_x));
  return true;
}

#ifndef MN_ROUTE_NARROW_CT
#define MN_ROUTE_NARROW_CT 16  // 8-channel tiles measured slower (1013 against 952 us at 48 x 48)
#endif
template <typename XT>
static bool launch_stencil(int variant, const void* x, int B, int T, int C, const mn_route_dims* d, int L, int k,
                           const RouteWs& ws, void* topk_x, cudaStream_t st) {
  const bool wide = (size_t)T * 32 * sizeof(float) <= 200 * 1024;
  constexpr int NCT = MN_ROUTE_NARROW_CT;
  if (variant == 1) {
    if (wide) return launch_stencil_ct<XT, 32, 2, 0>(x, B, T, C, d, L, k, ws, topk_x, st);
    else return launch_stencil_ct<XT, NCT, 2, 0>(x, B, T, C, d, L, k, ws, topk_x, st);
  } else if (variant == 2) {
    if (wide) return launch_stencil_ct<XT, 32, 1, -1>(x, B, T, C, d, L, k, ws, topk_x, st);
    else return launch_stencil_ct<XT, NCT, 1, -1>(x, B, T, C, d, L, k, ws, topk_x, st);
  } else {
    if (wide) return launch_stencil_ct<XT, 32, 0, -1>(x, B, T, C, d, L, k, ws, topk_x, st);
    else return launch_stencil_ct<XT, NCT, 0, -1>(x, B, T, C, d, L, k, ws, topk_x, st);
  }
}

// Banding for route_score_lane: receiver rows of a band in <= 110 KB of
// shared memory (two CTAs per SM).  Covers Cm in {32, 64} and kc <= 16.
static bool lane_score_plan(int Cm, int kc, int grid_h, int grid_w, int radius_rows, Banding* bd, size_t* smem) {
  if ((Cm != 32 && Cm != 64) || kc > kMaxKc) return false;
  const size_t budget = 110 * 1024;
  for (int nb = 1; nb <= grid_h; ++nb) {
    const int rows = (grid_h + nb - 1) / nb;
    const int need_rows = (nb == 1) ? grid_h : std::min(grid_h, rows + 2 * radius_rows);
    const size_t bytes = ((size_t)(need_rows * grid_w + 1) / 2 + 1) * (Cm + 4) * sizeof(float);
    if (bytes <= budget) {
      bd->bands = (grid_h + rows - 1) / rows;
      bd->rows = rows;
      bd->radius_rows = radius_rows;
      bd->cap = 0;
      *smem = bytes;
      return true;
    }
  }
  return false;
}

template <int MDT>
static bool launch_score_lane(const void* metrics, const int32_t* table, int B, int T, int Cm, int grid_w, int half,
                              int kc, int kin, const Banding& bd, size_t smem, float tau1, const RouteWs& ws, int L,
                              int* status, cudaStream_t st) {
  using ET = typename Elem<MDT>::T;
  auto kern = Cm == 64 ? route_score_lane_kernel<MDT, 64> : route_score_lane_kernel<MDT, 32>;
  if (!ensure_smem(kern, smem)) return false;
  kern<<<dim3(B * bd.bands, L), kLaneScoreThreads, smem, st>>>(static_cast<const ET*>(metrics), table, B, T, grid_w,
                                                               half, kc, kin, bd, tau1, ws, status);
  return true;
}

template <int MDT>
static bool launch_score(const void* metrics, const int32_t* table, int B, int T, int Cm, int grid_w,
                         int half, int kc, int kin, const Banding& bd, float tau1, const RouteWs& ws,
                         int L, int* status, cudaStream_t st) {
  using ET = typename Elem<MDT>::T;
  size_t smem = (size_t)bd.cap * Cm * sizeof(float);
  dim3 grid(B * bd.bands, L);
  if (!ensure_smem(route_score_kernel<MDT>, smem)) return false;
  route_score_kernel<MDT><<<grid, 512, smem, st>>>(static_cast<const ET*>(metrics), table, B, T, Cm,
                                                    grid_w, half, kc, kin, bd, tau1, ws, status);
  return true;
}

extern "C" int mn_route_and_gather(const mn_route_dims* dims, const int32_t* dev_table, int batch,
                                   int channels, int metric_dim, int num_layers, const int* r_list,
                                   int k, float tau1, float tau2, const void* x, int x_dtype,
                                   const void* metrics, int metric_dtype, void* workspace,
                                   size_t workspace_bytes, void* topk_x, float* topk_size,
                                   int64_t* topk_idx, float* size_out, float* center_out,
                                   int* status, void* stream) {
  if (!dims || !dev_table || !x || !metrics || !workspace || !topk_x || !topk_size || !topk_idx ||
      !size_out || !center_out || !r_list)
    return MN_ERR_ARG;
  if (batch <= 0 || channels <= 0 || metric_dim <= 0 || num_layers <= 0 || num_layers > 64)
    return MN_ERR_ARG;
  if (x_dtype < 0 || x_dtype > 2 || metric_dtype < 0 || metric_dtype > 2) return MN_ERR_ARG;
  const int half = dims->half, kc = dims->kc, kin = dims->kin;
  const int P = dims->num_patches, T = P + 1;
  if (P <= 0 || P % 2 != 0 || half * 2 != P || dims->grid_h * dims->grid_w != P) return MN_ERR_ARG;
  if (metric_dim > 128 || kc <= 0 || kc > 32 || kin <= 0 || k <= 0 || k > P) return MN_ERR_UNSUPPORTED;
  if (half > 4 * 512 || next_pow2(half) > 2048 * 4) return MN_ERR_UNSUPPORTED;  // route_mass: 4 receivers per thread
  if (mn_route_workspace_bytes(dims, batch, num_layers) > workspace_bytes) return MN_ERR_WORKSPACE;
  KBudget kb;
  for (int l = 0; l < num_layers; ++l) {
    int r = std::min(r_list[l], (T - 1) / 2);
    if (r <= 0) return MN_ERR_UNSUPPORTED;  // a no-op layer is not on the canonical path
    if (dims->valid_rows[l & 1] < r) return MN_INFEASIBLE_BUDGET;
    kb.v[l] = r;
  }
  const Banding bd = make_banding(dims->grid_h, dims->grid_w, dims->radius_rows, metric_dim);
  if (bd.bands <= 0) return MN_ERR_UNSUPPORTED;
  int ct = 32;
  while (ct > 8 && (size_t)T * ct * sizeof(float) > 200 * 1024) ct >>= 1;
  if ((size_t)T * ct * sizeof(float) > 220 * 1024) return MN_ERR_UNSUPPORTED;
  const int np_sel = next_pow2(half);
  const size_t smem_sel = row_scratch_bytes(np_sel) + (size_t)half * sizeof(float);
  const size_t smem_mass = mass_smem_bytes(T, k);
  if (smem_sel > 220 * 1024 || smem_mass > 220 * 1024 || kc > kMaxKc || next_pow2(P) > 8 * kMassThreads)
    return MN_ERR_UNSUPPORTED;

  cudaStream_t st = static_cast<cudaStream_t>(stream);
  float* f = static_cast<float*>(workspace);
  RouteWs ws;
  const size_t LBh = (size_t)num_layers * batch * half;
  ws.assign = f;   f += LBh * kc;
  ws.energy = f;   f += LBh;
  ws.asum = f;     f += LBh;
  ws.wa_old = f;   f += LBh;
  ws.wb_old = f;   f += LBh;
  ws.wb_safe = f;  f += LBh;
  ws.partials = f; f += (size_t)num_layers * batch * dims->grid_h * 2;
  ws.cf = f;       f += LBh * kStencilSlots;
  ws.carrier_tok = reinterpret_cast<int32_t*>(f);

  cudaGetLastError();  // clear any stale error so the check below is ours
  Banding lbd;
  size_t lsmem = 0;
  const bool lane = reinterpret_cast<uintptr_t>(metrics) % 16 == 0 &&  // 16-byte row loads
                    lane_score_plan(metric_dim, kc, dims->grid_h, dims->grid_w, dims->radius_rows, &lbd, &lsmem);
  const int bands_used = lane ? lbd.bands : bd.bands;
  bool ok;
  if (lane) {
    if (metric_dtype == MN_F16)
      ok = launch_score_lane<MN_F16>(metrics, dev_table, batch, T, metric_dim, dims->grid_w, half, kc, kin, lbd, lsmem, tau1, ws, num_layers, status, st);
    else if (metric_dtype == MN_BF16)
      ok = launch_score_lane<MN_BF16>(metrics, dev_table, batch, T, metric_dim, dims->grid_w, half, kc, kin, lbd, lsmem, tau1, ws, num_layers, status, st);
    else
      ok = launch_score_lane<MN_F32>(metrics, dev_table, batch, T, metric_dim, dims->grid_w, half, kc, kin, lbd, lsmem, tau1, ws, num_layers, status, st);
  } else if (metric_dtype == MN_F16) {
    ok = launch_score<MN_F16>(metrics, dev_table, batch, T, metric_dim, dims->grid_w, half, kc, kin, bd, tau1, ws, num_layers, status, st);
  } else if (metric_dtype == MN_BF16) {
    ok = launch_score<MN_BF16>(metrics, dev_table, batch, T, metric_dim, dims->grid_w, half, kc, kin, bd, tau1, ws, num_layers, status, st);
  } else {
    ok = launch_score<MN_F32>(metrics, dev_table, batch, T, metric_dim, dims->grid_w, half, kc, kin, bd, tau1, ws, num_layers, status, st);
  }
  if (!ok) return MN_ERR_LAUNCH;  // nothing launched: the driver refused a shared-memory size

  if (!ensure_smem(route_select_kernel, smem_sel) || !ensure_smem(route_mass_kernel, smem_mass))
    return MN_ERR_LAUNCH;
  route_select_kernel<<<dim3(batch, num_layers), kSelectThreads, smem_sel, st>>>(dev_table, batch, half, kc, kin,
                                                                                 bands_used, kb, tau2, ws, status);
  const int stencil = stencil_variant(dims);
  route_mass_kernel<<<batch, kMassThreads, smem_mass, st>>>(dev_table, batch, T, half, kc, kin, num_layers, k,
                                                            stencil > 0 ? 1 : 0, ws, size_out, center_out,
                                                            topk_size, topk_idx);

  if (stencil > 0) {
    if (x_dtype == MN_F16)
      ok = launch_stencil<__half>(stencil, x, batch, T, channels, dims, num_layers, k, ws, topk_x, st);
    else if (x_dtype == MN_BF16)
      ok = launch_stencil<__nv_bfloat16>(stencil, x, batch, T, channels, dims, num_layers, k, ws, topk_x, st);
    else
      ok = launch_stencil<float>(stencil, x, batch, T, channels, dims, num_layers, k, ws, topk_x, st);
  } else if (x_dtype == MN_F16) {
    ok = launch_transport<__half>(x, dev_table, batch, T, channels, half, kc, kin, num_layers, k, ws, topk_x, ct, st);
  } else if (x_dtype == MN_BF16) {
    ok = launch_transport<__nv_bfloat16>(x, dev_table, batch, T, channels, half, kc, kin, num_layers, k, ws, topk_x, ct, st);
  } else {
    ok = launch_transport<float>(x, dev_table, batch, T, channels, half, kc, kin, num_layers, k, ws, topk_x, ct, st);
  }
  if (!ok) return MN_ERR_LAUNCH;
  return cudaGetLastError() == cudaSuccess ? MN_OK : MN_ERR_LAUNCH;
}
