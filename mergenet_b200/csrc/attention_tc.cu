// Tensor-core (tcgen05 + TMEM) attention for head_dim 64, fp16 / bf16.
//
// One CTA of 128 threads owns 128 query rows of one (image, head); thread t
// owns row t, which is TMEM lane t of the accumulators.  Q, K and V tiles are
// brought into 128B-swizzled shared memory by TMA (one thread issues the
// bulk tensor copies, completion is counted on mbarriers), S = Q K^T is
// accumulated in TMEM by tcgen05.mma issued from one thread, each thread
// turns its S row into fp16 / bf16 probabilities in shared memory, and
// O = P V accumulates in TMEM.  The next block's S = Q K^T is issued right
// after this block's P.V, so it runs while the CTA finishes the block.
//
//   window >= 0: sliding window |i - j| <= window over one sequence (the
//     LocalAttention path, opentome/timm/bias_local_attn.py:486-625 / :243-483):
//     up to window 16 the 128 + 2*window keys of the tile form one block.
//   window <  0: every key (the recovery cross-attention core,
//     opentome/models/mergenet/model.py:173-188, and the latent blocks):
//     64-key blocks with an online softmax.
//
// Every wait is bounded; on timeout the CTA records an error bit and stops
// issuing work.
#include <algorithm>

#include "common.cuh"
#include "tc_common.cuh"
#include "tma.cuh"

namespace mn {

constexpr int kTcD = 64;
constexpr int kTcM = 128;

template <int NB>
struct TcSmem {
  // K is dead once S = Q K^T has completed, so one K buffer suffices; V is
  // read by P.V while the next block streams in, so the multi-block paths
  // (NB <= 128) keep two V stages.  NB = 128 / 160: ~97 KB, two CTAs per SM;
  // NB = 64: ~57 KB, three CTAs per SM.
  static constexpr int kStages = NB <= 128 ? 2 : 1;
  static constexpr int kTmemCols = NB + kTcD <= 128 ? 128 : 256;  // S then O
  static constexpr int kMinBlocks = NB == 64 ? 3 : 2;
  static constexpr int kPAtoms = (NB + 63) / 64;
  static constexpr uint32_t q_off = 0;
  static constexpr uint32_t k_off = q_off + kTcM * 128;
  static constexpr uint32_t kv_stage = NB * 128;
  static constexpr uint32_t v_off = k_off + kv_stage;
  static constexpr uint32_t p_off = (v_off + kStages * kv_stage + 1023) & ~1023u;
  static constexpr uint32_t bias_off = p_off + kPAtoms * kTcM * 128;  // two blocks' biases
  // barriers: S done, P.V done, Q landed, K landed, V stage 0 / 1 landed
  static constexpr uint32_t bar_off = bias_off + 2 * NB * 4;
  static constexpr uint32_t tmem_slot_off = bar_off + 6 * 8;
  static constexpr uint32_t bytes = tmem_slot_off + 8 + 1024;  // + alignment slack
};
static_assert(TcSmem<160>::bytes <= 113 * 1024 && TcSmem<128>::bytes <= 113 * 1024, "two CTAs per SM");
static_assert(TcSmem<64>::bytes <= 75 * 1024, "three CTAs per SM");

template <typename ET>
__device__ __forceinline__ uint4 pack8(const float* p) {
  uint4 r;
  uint32_t* w = reinterpret_cast<uint32_t*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    ET lo = from_f32<ET>(p[2 * i]), hi = from_f32<ET>(p[2 * i + 1]);
    w[i] = (uint32_t)(*reinterpret_cast<uint16_t*>(&lo)) | ((uint32_t)(*reinterpret_cast<uint16_t*>(&hi)) << 16);
  }
  return r;
}

__device__ __forceinline__ float fast_ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <typename ET>
__device__ __forceinline__ uint32_t pack2(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Log2-domain growth of a row maximum that is absorbed without rescaling O:
// probabilities then reach at most 2^8, well inside fp16 / bf16 range, and O
// and the row sum share the same stale maximum, so the result is unchanged.
constexpr float kRescaleLog2 = 8.0f;

// NCH: S chunks (32 columns) a warp can need in one block.  With a window
// the legal keys of a warp's 32 rows span at most 32 + 2*window columns, so
// NB = 160 (window <= 16) needs at most three chunks; otherwise all.
template <int NB>
struct TcChunks {
  static constexpr int kAll = NB / 32;
  static constexpr int kWarp = NB == 160 ? 3 : kAll;
};

// The CLS row of the LocalAttention block (row 0 attends to every key,
// opentome/timm/bias_local_attn.py:704-719), computed by the CTA that owns
// query tile 0 after its windowed rows: scores q0 . k_j * scale (+ bias_j),
// softmax exp(s - max) / sum, then sum_j p_j v_j with 16-byte value loads
// (8 threads per value row, 16 rows in flight).  `scratch` holds the scores
// (Nk floats) and the partial sums; qrow is the CLS query (global memory).
template <typename ET>
__device__ void cls_row_global(const ET* __restrict__ qrow, const ET* __restrict__ kg, const ET* __restrict__ vg,
                               int64_t kb, int64_t kn, int64_t kh, int b, int h, int Nq, int Nk, int H, float scale,
                               const void* __restrict__ bias, int bias_dtype, float* scratch, void* out,
                               int out_dtype) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float* sp = scratch;                         // [Nk]
  float* qv = sp + ((Nk + 3) & ~3);            // [64]
  float* part = qv + kTcD;                     // [16][64]
  float* red = part + 16 * kTcD;               // [8]
  if (tid < kTcD) qv[tid] = to_f32(qrow[tid]);
  __syncthreads();
  const ET* kbh = kg + (int64_t)b * kb + (int64_t)h * kh;
  const ET* vbh = vg + (int64_t)b * kb + (int64_t)h * kh;
  float mx = -INFINITY;
  auto score = [&](int j, const uint4* u) {
    float acc0 = 0.f, acc1 = 0.f;  // even / odd 8-channel groups
#pragma unroll
    for (int c = 0; c < kTcD / 8; ++c) {
      const ET* e = reinterpret_cast<const ET*>(u + c);
      float a = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) a = fmaf(qv[c * 8 + i], to_f32(e[i]), a);
      if (c & 1) acc1 += a; else acc0 += a;
    }
    float sc = (acc0 + acc1) * scale;
    if (bias) sc += to_f32(from_f32<ET>(load_any(bias, bias_dtype, (int64_t)b * Nk + j)));
    sp[j] = sc;
    mx = fmaxf(mx, sc);
  };
  int j = tid;
  for (; j + (int)blockDim.x < Nk; j += 2 * blockDim.x) {  // two keys' rows in flight
    uint4 u[2][kTcD / 8];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const uint4* kr = reinterpret_cast<const uint4*>(kbh + (int64_t)(j + r * blockDim.x) * kn);
#pragma unroll
      for (int c = 0; c < kTcD / 8; ++c) u[r][c] = __ldg(kr + c);
    }
    score(j, u[0]);
    score(j + blockDim.x, u[1]);
  }
  if (j < Nk) {
    uint4 u[kTcD / 8];
    const uint4* kr = reinterpret_cast<const uint4*>(kbh + (int64_t)j * kn);
#pragma unroll
    for (int c = 0; c < kTcD / 8; ++c) u[c] = __ldg(kr + c);
    score(j, u);
  }
  mx = warp_max(mx);
  if (lane == 0) red[warp] = mx;
  __syncthreads();
  mx = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
  float sum = 0.f;
  for (int j = tid; j < Nk; j += blockDim.x) {
    const float e = expf(sp[j] - mx);
    sp[j] = e;
    sum += e;
  }
  sum = warp_sum(sum);
  __syncthreads();  // every thread has read red[] and written its p_j
  if (lane == 0) red[4 + warp] = sum;
  __syncthreads();
  const float tot = (red[4] + red[5]) + (red[6] + red[7]);
  const int sub = tid & 7, rg = tid >> 3;  // 8 threads per value row, 16 rows in flight
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  auto accumulate = [&](int jj, const uint4& u) {
    const ET* e = reinterpret_cast<const ET*>(&u);
    const float pj = sp[jj];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = fmaf(pj, to_f32(e[i]), acc[i]);
  };
  int jv = rg;
  for (; jv + 48 < Nk; jv += 64) {  // four value rows in flight per thread
    uint4 u[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) u[r] = __ldg(reinterpret_cast<const uint4*>(vbh + (int64_t)(jv + 16 * r) * kn) + sub);
#pragma unroll
    for (int r = 0; r < 4; ++r) accumulate(jv + 16 * r, u[r]);
  }
  for (; jv < Nk; jv += 16) accumulate(jv, __ldg(reinterpret_cast<const uint4*>(vbh + (int64_t)jv * kn) + sub));
#pragma unroll
  for (int i = 0; i < 8; ++i) part[rg * kTcD + sub * 8 + i] = acc[i];
  __syncthreads();
  if (tid < kTcD) {
    float o = 0.f;
    for (int g = 0; g < 16; ++g) o += part[g * kTcD + tid];
    store_any(out, out_dtype, ((int64_t)b * Nq * H + h) * kTcD + tid, o / tot);
  }
}

// Largest key count whose CLS scratch fits the P tile of the NB-key kernel.
template <int NB>
constexpr int cls_max_keys() {
  return (int)((TcSmem<NB>::kPAtoms * kTcM * 128) / 4) - (kTcD + 16 * kTcD + 8) - 4;
}

__device__ __forceinline__ void prefetch_rows(const CUtensorMap* map, int order, int h, int n, int b) {
  if (order == 0)
    tma::prefetch_l2_4d(map, 0, h, n, b);
  else
    tma::prefetch_l2_4d(map, 0, n, h, b);
}

// WIN: sliding window (per-row key ranges, masked per element).  Without a
// window every row sees the same keys, so keys past the end get a -inf bias
// and no element is masked.  BIAS: a per-key bias is given.
// Tile coordinates of a (d, h, n, b) tensor map: order 0 has heads before
// tokens in the map's dimension list (packed-qkv / BNHD layouts), order 1
// tokens before heads (BHND).
__device__ __forceinline__ void load_rows(uint32_t dst, const CUtensorMap* map, int order, int h, int n, int b,
                                          uint64_t* bar) {
  if (order == 0)
    tma::load_4d(dst, map, 0, h, n, b, bar);
  else
    tma::load_4d(dst, map, 0, n, h, b, bar);
}

// WIN: sliding window (per-row key ranges, masked per element).  Without a
// window every row sees the same keys, so keys past the end get a -inf bias
// and no element is masked.  BIAS: a per-key bias is given.
template <typename ET, int NB, bool WIN, bool BIAS>
__global__ void __launch_bounds__(128, TcSmem<NB>::kMinBlocks) attn_tc_kernel(
    const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
    const __grid_constant__ CUtensorMap tm_v, int q_order, int kv_order, int Nq, int Nk, int H, int window,
    float scale, const void* __restrict__ bias, int bias_dtype, void* __restrict__ out, int out_dtype,
    int* __restrict__ err, int cls_global, const ET* __restrict__ qg, int64_t qb, int64_t qh,
    const ET* __restrict__ kg, const ET* __restrict__ vg, int64_t kb, int64_t kn, int64_t kh) {
  using S = TcSmem<NB>;
  constexpr int NCH = TcChunks<NB>::kWarp;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sq = base + S::q_off;
  uint8_t* sk = base + S::k_off;
  uint8_t* sv = base + S::v_off;
  uint8_t* sp = base + S::p_off;
  float* sbias2 = reinterpret_cast<float*>(base + S::bias_off);  // [2][NB]
  uint64_t* bar = reinterpret_cast<uint64_t*>(base + S::bar_off);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base + S::tmem_slot_off);

  const int tid = threadIdx.x, warp = tid >> 5;
  const int q0 = blockIdx.x * kTcM, h = blockIdx.y, b = blockIdx.z;
  constexpr int ab_bf16 = std::is_same<ET, __nv_bfloat16>::value ? 1 : 0;
  constexpr uint32_t idesc_o = tc::idesc_f16(ab_bf16, 1, kTcM, kTcD);
  const float kLog2e = 1.4426950408889634f;
  const float sl2 = scale * kLog2e;  // scores enter the softmax in log2 units

  uint64_t* bar_s = bar;      // arrives when S = Q K^T (and all earlier MMAs) completed
  uint64_t* bar_o = bar + 1;  // arrives when P.V (and all earlier MMAs) completed
  uint64_t* bar_q = bar + 2;  // Q tile landed
  uint64_t* bar_k = bar + 3;  // K block landed (one phase per block)
  uint64_t* bar_v = bar + 4;  // V stage landed: [0], [1]
  int klo = 0, khi = Nk;
  if (WIN) {
    klo = max(0, q0 - window);
    khi = min(Nk, q0 + kTcM + window);
  }
  const int nblocks = (khi - klo + NB - 1) / NB;

  // the per-key bias (log2 units) of block blk into its buffer; without a
  // window, keys past the end get -inf
  auto stage_bias = [&](int blk) {
    if (BIAS || !WIN) {
      const int kstart = klo + blk * NB;
      const int kvalid = min(NB, khi - kstart);
      float* sb = sbias2 + (blk & 1) * NB;
      for (int j = tid; j < NB; j += blockDim.x) {
        float bv = WIN ? 0.f : -INFINITY;
        if (j < kvalid) {
          bv = 0.f;
          if (BIAS) bv = to_f32(from_f32<ET>(load_any(bias, bias_dtype, (int64_t)b * Nk + kstart + j))) * kLog2e;
        }
        sb[j] = bv;
      }
    }
  };
  // S = Q K^T for block blk, issued by thread 0 once K has landed
  auto issue_s = [&](int blk, uint32_t t_s) -> bool {
    if (!tc::mbar_wait(bar_k, blk & 1, err)) return false;
    tc::fence_after_sync();
    const int kvalid = min(NB, khi - (klo + blk * NB));
    const int kpad = (kvalid + 31) & ~31;
    // a 16-wide K step moves the descriptors' start-address field (address
    // >> 4) by 32 bytes >> 4 = 2
    const uint64_t dq = tc::sw128_desc(tc::smem_u32(sq), 16), dk = tc::sw128_desc(tc::smem_u32(sk), 16);
    const uint32_t idesc_s = tc::idesc_f16(ab_bf16, 0, kTcM, kpad);
#pragma unroll
    for (int kk = 0; kk < kTcD / 16; ++kk) tc::mma_f16_ss(t_s, dq + 2 * kk, dk + 2 * kk, idesc_s, kk > 0);
    tc::mma_commit(bar_s);
    return true;
  };

  if (warp == 0) tc::tmem_alloc(tmem_slot, S::kTmemCols);
  if (tid == 0) {
    for (int i = 0; i < 6; ++i) tc::mbar_init(bar + i, 1);
    tc::fence_mbar_init();
    tma::prefetch_map(&tm_q);
    tma::prefetch_map(&tm_k);
    tma::prefetch_map(&tm_v);
    if (nblocks > 0) {
      // Q and the first K/V block in flight together
      tma::expect_tx(bar_q, kTcM * 128);
      load_rows(tc::smem_u32(sq), &tm_q, q_order, h, q0, b, bar_q);
      tma::expect_tx(bar_k, NB * 128);
      load_rows(tc::smem_u32(sk), &tm_k, kv_order, h, klo, b, bar_k);
      tma::expect_tx(bar_v, NB * 128);
      load_rows(tc::smem_u32(sv), &tm_v, kv_order, h, klo, b, bar_v);
    }
  }
  if (nblocks > 0) stage_bias(0);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  const uint32_t t_s = tmem, t_o = tmem + NB;
  const uint32_t lane_sel = (uint32_t)(warp * 32) << 16;
  bool ok = true;
  if (tid == 0 && nblocks > 0) {
    ok = tc::mbar_wait(bar_q, 0, err) && issue_s(0, t_s);
    if (!ok && err) atomicOr(err, MN_STATUS_TC_TIMEOUT);
  }

  const int qi = q0 + tid;  // this thread's query row
  const bool live = WIN || q0 + warp * 32 < Nq;  // warp-uniform
  float m_run = -INFINITY, l_run = 0.f;
  // the last phase issued on each copy barrier, for the exit drain
  int k_issued = nblocks > 0 ? 0 : -1, v_issued[2] = {nblocks > 0 ? 0 : -1, -1};

  for (int blk = 0; blk < nblocks && ok; ++blk) {
    const int kstart = klo + blk * NB;
    const int kvalid = min(NB, khi - kstart);  // keys of this block
    // MMA extent: whole 32-column chunks, so every S column the softmax
    // reads was written by this block's MMA
    const int kpad = (kvalid + 31) & ~31;
    const int stage = blk % S::kStages;
    const float* sbias = sbias2 + (blk & 1) * NB;
    // every S commit is waited for, in order: phase blk of bar_s
    ok = tc::mbar_wait(bar_s, blk & 1, err);
    if (!ok) break;
    tc::fence_after_sync();
    // S done -- and with it every earlier MMA, including the previous P.V --
    // so K and the other V stage are free: fetch the next block while this
    // block's softmax runs
    if (blk + 1 < nblocks) {
      // the K and V copies are issued from warps 1 and 2, so neither issue
      // latency adds to warp 0's (which issues the MMAs)
      const int ns = (blk + 1) % S::kStages;
      if (tid == 32) {
        tma::expect_tx(bar_k, NB * 128);
        load_rows(tc::smem_u32(sk), &tm_k, kv_order, h, kstart + NB, b, bar_k);
      } else if (tid == 64) {
        tma::expect_tx(bar_v + ns, NB * 128);
        load_rows(tc::smem_u32(sv + ns * S::kv_stage), &tm_v, kv_order, h, kstart + NB, b, bar_v + ns);
      }
      k_issued = blk + 1;  // tracked by every thread: thread 0 drains at exit
      v_issued[ns] = blk + 1;
      stage_bias(blk + 1);
    }

    // this row's legal keys, relative to the block: [jlo, jhi)
    int jlo = 0, jhi = kvalid;
    int c_lo = 0, nch = kpad >> 5;  // without a window: every chunk, every row
    if (WIN) {
      jlo = max(jlo, qi - window - kstart);
      jhi = min(jhi, qi + window + 1 - kstart);
      if (qi >= Nq) jhi = jlo;  // padding rows: no keys
      // the warp's column chunks that can hold a legal key: [c_lo, c_lo + nch).
      // Rows without a key in this block (jlo >= jhi; jlo may lie past the
      // block) take no part, so 0 <= wlo and whi <= kvalid <= NB.
      const bool has = jlo < jhi;
      const int wlo = (int)__reduce_min_sync(0xffffffffu, (unsigned)(has ? jlo : NB));
      const int whi = (int)__reduce_max_sync(0xffffffffu, (unsigned)(has ? jhi : 0));
      c_lo = min(wlo >> 5, TcChunks<NB>::kAll);
      nch = whi > wlo ? ((whi + 31) >> 5) - c_lo : 0;
    }
    // never past the S tile: c_lo + nch <= NB / 32 (and at most NCH chunks)
    if (nch > NCH || c_lo + nch > TcChunks<NB>::kAll) {  // cannot happen, see above
      nch = max(0, min(NCH, TcChunks<NB>::kAll - c_lo));
      if (err && (tid & 31) == 0) atomicOr(err, MN_STATUS_TC_TIMEOUT);
    }

    // a warp whose 32 rows all lie past the last query (the tail tile) has
    // nothing to compute; its P rows feed only O rows that are never stored
    if (live) {
      // S rows of the warp's chunks, all loads in flight before one wait
      float sc[NCH * 32];
#pragma unroll
      for (int u = 0; u < NCH; ++u)
        if (u < nch) tc::tmem_ld32_nowait(t_s + lane_sel + (c_lo + u) * 32, sc + u * 32);
      tc::tmem_ld_wait<NCH * 32>(sc);

      // pass 1: log2-domain logits (illegal keys -inf) and the row maximum
      float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int u = 0; u < NCH; ++u) {
        if (u >= nch) continue;
        const int cb = (c_lo + u) * 32;
        const bool whole = !WIN || __all_sync(0xffffffffu, jlo <= cb && jhi >= cb + 32);
        const float4* b4 = reinterpret_cast<const float4*>(sbias + cb);
        if (whole) {
#pragma unroll
          for (int i4 = 0; i4 < 8; ++i4) {
            float4 bb = make_float4(0.f, 0.f, 0.f, 0.f);
            if (BIAS || !WIN) bb = b4[i4];
            const float bv[4] = {bb.x, bb.y, bb.z, bb.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              float& x = sc[u * 32 + i4 * 4 + e];
              x = fmaf(x, sl2, bv[e]);
              mx4[e] = fmaxf(mx4[e], x);
            }
          }
        } else {
#pragma unroll
          for (int i4 = 0; i4 < 8; ++i4) {
            float4 bb = make_float4(0.f, 0.f, 0.f, 0.f);
            if (BIAS) bb = b4[i4];
            const float bv[4] = {bb.x, bb.y, bb.z, bb.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int j = cb + i4 * 4 + e;
              float& x = sc[u * 32 + i4 * 4 + e];
              x = (j >= jlo && j < jhi) ? fmaf(x, sl2, bv[e]) : -INFINITY;
              mx4[e] = fmaxf(mx4[e], x);
            }
          }
        }
      }
      const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
      const float m_new = fmaxf(m_run, mx);
      // keep the running maximum unless it grew by more than 2^8
      const float m_use = (m_run == -INFINITY || m_new - m_run > kRescaleLog2) ? m_new : m_run;
      const float corr = (m_run == -INFINITY || m_use == m_run) ? 1.f : fast_ex2(m_run - m_use);
      const float msub = m_use == -INFINITY ? 0.f : m_use;

      // pass 2: probabilities -> P in shared memory; chunks outside the warp's
      // range are zero
      float ls4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int u = 0; u < NCH; ++u) {
        if (u >= nch) continue;
        const int c = c_lo + u;
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          uint4 pk;
          uint32_t* w = reinterpret_cast<uint32_t*>(&pk);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float p0 = fast_ex2(sc[u * 32 + g * 8 + 2 * e] - msub);
            const float p1 = fast_ex2(sc[u * 32 + g * 8 + 2 * e + 1] - msub);
            ls4[(2 * e) & 3] += p0;
            ls4[(2 * e + 1) & 3] += p1;
            w[e] = pack2<ET>(p0, p1);
          }
          const int key8 = c * 4 + g;  // 8-key chunk index
          *reinterpret_cast<uint4*>(sp + (key8 >> 3) * (kTcM * 128) + tc::sw128_off(tid, key8 & 7)) = pk;
        }
      }
      const int c_end = (kpad + 31) >> 5;  // chunks the P.V MMA reads
      for (int c = 0; c < c_end; ++c) {
        if (c >= c_lo && c < c_lo + nch) continue;
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          const int key8 = c * 4 + g;
          *reinterpret_cast<uint4*>(sp + (key8 >> 3) * (kTcM * 128) + tc::sw128_off(tid, key8 & 7)) =
              make_uint4(0u, 0u, 0u, 0u);
        }
      }
      // rescale the running output rows (warp-collective TMEM access: the
      // whole warp takes part when any of its rows needs it)
      if (blk > 0 && __any_sync(0xffffffffu, corr != 1.f)) {
        float o[32];
#pragma unroll
        for (int c = 0; c < kTcD / 32; ++c) {
          tc::tmem_ld32(t_o + lane_sel + c * 32, o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] *= corr;
          tc::tmem_st32(t_o + lane_sel + c * 32, o);
        }
      }
      l_run = l_run * corr + ((ls4[0] + ls4[1]) + (ls4[2] + ls4[3]));
      m_run = m_use;
    }
    tc::fence_async_smem();
    tc::fence_before_sync();
    __syncthreads();
    if (tid == 0) {
      tc::fence_after_sync();
      // P.V once this block's V stage has landed, then the next block's S
      if (!tc::mbar_wait(bar_v + stage, (blk / S::kStages) & 1, err)) {
        ok = false;
      } else {
        // P: 32 bytes per K step inside a 64-key atom, 16 KB between atoms;
        // V: 16 key rows (2 KB) per K step
        const uint64_t dp = tc::sw128_desc(tc::smem_u32(sp), 16);
        const uint64_t dv = tc::sw128_desc(tc::smem_u32(sv + stage * S::kv_stage), 16384);
        const int nsteps = kpad / 16;
#pragma unroll
        for (int kk = 0; kk < NB / 16; ++kk)  // unrolled: descriptor offsets are constants
          if (kk < nsteps)
            tc::mma_f16_ss(t_o, dp + (uint64_t)((kk >> 2) * (kTcM * 128 / 16) + (kk & 3) * 2), dv + 128 * kk,
                           idesc_o, (blk > 0 || kk > 0) ? 1u : 0u);
        tc::mma_commit(bar_o);
        if (blk + 1 < nblocks) ok = issue_s(blk + 1, t_s);
      }
      if (!ok && err) atomicOr(err, MN_STATUS_TC_TIMEOUT);
    }
  }
  if (tid == 0) {
    // every bulk copy issued has landed before the CTA may exit
    if (k_issued >= 0) tc::mbar_wait(bar_k, k_issued & 1, nullptr);
    for (int st = 0; st < S::kStages; ++st)
      if (v_issued[st] >= 0) tc::mbar_wait(bar_v + st, (v_issued[st] / S::kStages) & 1, nullptr);
    if (nblocks > 0) tc::mbar_wait(bar_q, 0, nullptr);
  }
  if (ok && nblocks > 0) {
    // bar_o is only waited for here, after its last arrival: the phase of the
    // final P.V has parity (nblocks - 1) & 1
    ok = tc::mbar_wait(bar_o, (nblocks - 1) & 1, err);
    tc::fence_after_sync();
  }
  if (ok && nblocks > 0) {
    const float inv = l_run > 0.f ? 1.0f / l_run : 0.f;
    const int64_t obase = (((int64_t)b * Nq + qi) * H + h) * kTcD;
#pragma unroll
    for (int c = 0; c < kTcD / 32; ++c) {
      if (!live) break;
      float o[32];
      tc::tmem_ld32(t_o + lane_sel + c * 32, o);  // warp-collective: every row loads
      if (qi >= Nq) continue;
#pragma unroll
      for (int i = 0; i < 32; ++i) o[i] *= inv;
      if (out_dtype == MN_F32) {
        float4* dst = reinterpret_cast<float4*>(static_cast<float*>(out) + obase + c * 32);
#pragma unroll
        for (int i = 0; i < 8; ++i) dst[i] = make_float4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
      } else if (out_dtype == MN_F16) {
        uint4* dst = reinterpret_cast<uint4*>(static_cast<__half*>(out) + obase + c * 32);
#pragma unroll
        for (int i = 0; i < 4; ++i) dst[i] = pack8<__half>(o + 8 * i);
      } else {
        uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(out) + obase + c * 32);
#pragma unroll
        for (int i = 0; i < 4; ++i) dst[i] = pack8<__nv_bfloat16>(o + 8 * i);
      }
    }
  }
  if (!ok && tid == 0 && err) atomicOr(err, MN_STATUS_TC_TIMEOUT);
  tc::fence_before_sync();
  const int all_ok = __syncthreads_and(ok ? 1 : 0);  // a barrier with a CTA-uniform verdict
  if (warp == 0) tc::tmem_dealloc(tmem, S::kTmemCols);
  // the CLS row over every key, by the CTA of query tile 0 (its windowed row
  // 0 was written above and is replaced); every MMA has completed, so the P
  // tile is free scratch
  if (WIN && cls_global && q0 == 0 && all_ok && nblocks > 0)
    cls_row_global<ET>(qg + (int64_t)b * qb + (int64_t)h * qh, kg, vg, kb, kn, kh, b, h, Nq, Nk, H, scale, bias,
                       bias_dtype, reinterpret_cast<float*>(sp), out, out_dtype);
}

// ---------------------------------------------------------------------------
// CLS row of the windowed attention, folded into the persistent kernel.
// Query 0 attends every key (bias_local_attn.py:704-719).  The CTA that
// processes a (head, image)'s first query tile owns its CLS row: while a tile's
// K/V rows sit in shared memory, each warp scores the CLS query against 32 of
// the tile's own 128 keys and folds them into its running softmax state (max,
// sum, 64 outputs; log2 domain) held in shared memory.  The four warps' states
// are merged and row 0 is written after the last tile.  When the CTA's range
// of tiles ends before the (head, image) does, the rest of the keys are read
// from global memory.
// ---------------------------------------------------------------------------
constexpr int kClsState = 2 + kTcD;                               // max, sum, outputs
constexpr int kClsFloats = 2 * kTcD + 2 * 4 * kClsState;          // two queries, two sets of 4 warp states
constexpr uint32_t kClsBytes = kClsFloats * 4;

template <typename ET>
__device__ __forceinline__ float dot8(const uint4& u, const float* __restrict__ q) {
  const ET* e = reinterpret_cast<const ET*>(&u);
  const float4 qa = *reinterpret_cast<const float4*>(q), qb = *reinterpret_cast<const float4*>(q + 4);
  float a = to_f32(e[0]) * qa.x;
  a = fmaf(to_f32(e[1]), qa.y, a);
  a = fmaf(to_f32(e[2]), qa.z, a);
  a = fmaf(to_f32(e[3]), qa.w, a);
  float b = to_f32(e[4]) * qb.x;
  b = fmaf(to_f32(e[5]), qb.y, b);
  b = fmaf(to_f32(e[6]), qb.z, b);
  b = fmaf(to_f32(e[7]), qb.w, b);
  return a + b;
}

// Lane l's CLS logits (log2 domain) for key l of G groups of 32 keys each
// (group g: nv[g] valid keys; -inf past them).  Keys come from the swizzled
// K tile (row row0 + l, G = 1) or, when GLOBAL, from global rows
// key0 + g * gstride + l.  `bl2[g]` is the key's bias.
template <typename ET, bool GLOBAL, int G>
__device__ __forceinline__ void cls_warp_score(const float* __restrict__ qc, const int* nv, const uint8_t* sk,
                                               int row0, const ET* __restrict__ kbh, int64_t kn, int key0,
                                               int gstride, float sl2, const float* bl2, float* s) {
  const int lane = threadIdx.x & 31;
  uint4 kr[G][kTcD / 8];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    // tile rows past the valid keys are in bounds (zero-filled): read them
    // unconditionally and mask afterwards; a global row is clamped to its
    // group's last key, and an empty group reads nothing
    if (GLOBAL && nv[g] <= 0) continue;
    const int r = GLOBAL ? key0 + g * gstride + min(lane, nv[g] - 1) : 0;
#pragma unroll
    for (int c = 0; c < kTcD / 8; ++c)
      kr[g][c] = GLOBAL ? __ldg(reinterpret_cast<const uint4*>(kbh + (int64_t)r * kn) + c)
                        : *reinterpret_cast<const uint4*>(sk + tc::sw128_off(row0 + lane, c));
  }
#pragma unroll
  for (int g = 0; g < G; ++g) {
    if (GLOBAL && nv[g] <= 0) {
      s[g] = -INFINITY;
      continue;
    }
    float a0 = 0.f, a1 = 0.f;
#pragma unroll
    for (int c = 0; c < kTcD / 8; ++c) {
      if (c & 1) a1 += dot8<ET>(kr[g][c], qc + c * 8);
      else a0 += dot8<ET>(kr[g][c], qc + c * 8);
    }
    s[g] = lane < nv[g] ? fmaf(a0 + a1, sl2, bl2[g]) : -INFINITY;
  }
}

__device__ __forceinline__ float warp_max_f32(float v) {  // one warp-wide reduction instruction
  float r;
  asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(r) : "f"(v));
  return r;
}

// One warp folds its G scored groups (logit s[g] in lane l) into its CLS
// state, kept in registers: the running max m (warp-uniform), this lane's
// share l of the running sum, and this lane's unreduced share o[8] of the 64
// outputs (fresh: the state is empty).  For P.V lane (ks = l >> 3, dg = l & 7)
// takes keys ks*8 .. ks*8+7 of each group and channels dg*8 .. dg*8+7, from
// the swizzled V tile (rows row0 + key, G = 1) or, when GLOBAL, global rows
// key0 + g * gstride + key.
template <typename ET, bool GLOBAL, int G>
__device__ __forceinline__ void cls_warp_fold(const float* s, float& m, float& l, float* o, bool fresh, const int* nv,
                                              const uint8_t* sv, int row0, const ET* __restrict__ vbh, int64_t kn,
                                              int key0, int gstride) {
  const int lane = threadIdx.x & 31;
  const float m_old = fresh ? -INFINITY : m;
  float lm = s[0];
#pragma unroll
  for (int g = 1; g < G; ++g) lm = fmaxf(lm, s[g]);
  const float m_new = fmaxf(m_old, warp_max_f32(lm));
  const float msub = m_new == -INFINITY ? 0.f : m_new;
  const float alpha = fast_ex2(m_old - msub);
  float p[G], ps = 0.f;
#pragma unroll
  for (int g = 0; g < G; ++g) {
    p[g] = lane < nv[g] ? fast_ex2(s[g] - msub) : 0.f;
    ps += p[g];
  }
  l = fresh ? ps : fmaf(l, alpha, ps);
  m = m_new;
  const int ks = lane >> 3, dg = lane & 7;
#pragma unroll
  for (int k2 = 0; k2 < 8; ++k2) o[k2] = fresh ? 0.f : o[k2] * alpha;
  uint4 vr[G][8];
#pragma unroll
  for (int g = 0; g < G; ++g) {  // every row in flight; p = 0 past the valid keys
    if (GLOBAL && nv[g] <= 0) continue;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int kk = ks * 8 + i;
      vr[g][i] = GLOBAL ? __ldg(reinterpret_cast<const uint4*>(vbh + (int64_t)(key0 + g * gstride + min(kk, nv[g] - 1)) *
                                                                         kn) + dg)
                        : *reinterpret_cast<const uint4*>(sv + tc::sw128_off(row0 + kk, dg));
    }
  }
#pragma unroll
  for (int g = 0; g < G; ++g) {
    if (GLOBAL && nv[g] <= 0) continue;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float pk = __shfl_sync(0xffffffffu, p[g], ks * 8 + i);
      const ET* e = reinterpret_cast<const ET*>(&vr[g][i]);
#pragma unroll
      for (int k2 = 0; k2 < 8; ++k2) o[k2] = fmaf(pk, to_f32(e[k2]), o[k2]);
    }
  }
}

// Reduce a warp's register CLS state and store it to `st` = {max, sum, 64
// outputs} for the cross-warp merge.
__device__ __forceinline__ void cls_warp_publish(float m, float l, const float* o, float* st) {
  const int lane = threadIdx.x & 31;
  const float lsum = warp_sum(l);
  float r[8];
#pragma unroll
  for (int k2 = 0; k2 < 8; ++k2) {
    r[k2] = o[k2] + __shfl_xor_sync(0xffffffffu, o[k2], 8);
    r[k2] += __shfl_xor_sync(0xffffffffu, r[k2], 16);
  }
  if (lane < 8) {
#pragma unroll
    for (int k2 = 0; k2 < 8; ++k2) st[2 + lane * 8 + k2] = r[k2];
  }
  if (lane == 0) {
    st[0] = m;
    st[1] = lsum;
  }
}

// ---------------------------------------------------------------------------
// Windowed attention (window <= 16: one 160-key band per 128-query tile),
// persistent: CTA c walks an equal, contiguous range of tiles in (tile, head,
// image) order.  The next tile's Q is fetched as soon as this tile's
// S = Q K^T has completed, its K once the softmax is done (at once when there
// is no CLS row to fold in) and its V as soon as P.V has completed, so copy
// latency overlaps the softmax and epilogue; TMEM, barriers and tensor-map
// prefetches are set up once per CTA.  Copies are issued from warps 1-3 and
// the MMAs from thread 0.  OTMA: the O tile (16-bit) is staged in the V
// stage and written by one bulk tensor store instead of one 128-byte row
// per thread; the next V copy follows once the store has read the stage.
// ---------------------------------------------------------------------------
template <typename ET, bool BIAS, bool OTMA>
__global__ void __launch_bounds__(128, 2) attn_win_persistent_kernel(
    const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
    const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o, int q_order, int kv_order,
    int o_order, int N, int H, int B, int window, float scale, const void* __restrict__ bias,
    int bias_dtype, void* __restrict__ out, int out_dtype, int* __restrict__ err, int cls_global,
    const ET* __restrict__ qg, int64_t qb, int64_t qh, const ET* __restrict__ kg, const ET* __restrict__ vg,
    int64_t kb, int64_t kn, int64_t kh) {
  constexpr int NB = 160;
  using S = TcSmem<NB>;
  constexpr int NCH = TcChunks<NB>::kWarp;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sq = base + S::q_off;
  uint8_t* sk = base + S::k_off;
  uint8_t* sv = base + S::v_off;
  uint8_t* sp = base + S::p_off;
  float* sbias2 = reinterpret_cast<float*>(base + S::bias_off);  // [2][NB]
  uint64_t* bar = reinterpret_cast<uint64_t*>(base + S::bar_off);
  uint64_t* bar_s = bar;
  uint64_t* bar_o = bar + 1;
  uint64_t* bar_q = bar + 2;
  uint64_t* bar_k = bar + 3;
  uint64_t* bar_v = bar + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base + S::tmem_slot_off);
  float* cls_q = reinterpret_cast<float*>(base + ((S::tmem_slot_off + 8 + 15) & ~15u));  // [2][64]
  float* cls_st = cls_q + 2 * kTcD;                                                      // [2][4][kClsState]

  const int tid = threadIdx.x, warp = tid >> 5;
  constexpr int ab_bf16 = std::is_same<ET, __nv_bfloat16>::value ? 1 : 0;
  constexpr uint32_t idesc_o = tc::idesc_f16(ab_bf16, 1, kTcM, kTcD);
  const float kLog2e = 1.4426950408889634f;
  const float sl2 = scale * kLog2e;
  const int ntq = (N + kTcM - 1) / kTcM;
  const int total = ntq * H * B;
  // this CTA's tiles [t_begin, t_end)
  const int per = total / (int)gridDim.x, extra = total % (int)gridDim.x;
  const int t_begin = (int)blockIdx.x * per + min((int)blockIdx.x, extra);
  const int t_end = t_begin + per + ((int)blockIdx.x < extra ? 1 : 0);
  const bool late_k = cls_global != 0;  // K is read by the CLS fold until the softmax barrier

  struct Tile {
    int q0, h, b, klo, khi, qt, unit;
  };
  auto tile_of = [&](int t) {
    Tile x;
    x.qt = t % ntq;
    x.unit = t / ntq;
    x.q0 = x.qt * kTcM;
    x.h = x.unit % H;
    x.b = x.unit / H;
    x.klo = max(0, x.q0 - window);
    x.khi = min(N, x.q0 + kTcM + window);
    return x;
  };
  auto stage_bias = [&](const Tile& x, int buf) {
    if (BIAS) {
      float* sb = sbias2 + buf * NB;
      for (int j = tid; j < NB; j += blockDim.x) {
        float bv = 0.f;
        if (x.klo + j < x.khi)
          bv = to_f32(from_f32<ET>(load_any(bias, bias_dtype, (int64_t)x.b * N + x.klo + j))) * kLog2e;
        sb[j] = bv;
      }
    }
  };
  auto cls_combine = [&](const float* s0, int b, int h) {  // merge the four warps' states into row 0
    if (tid < kTcD) {
      float m = -INFINITY;
#pragma unroll
      for (int w = 0; w < 4; ++w) m = fmaxf(m, s0[w * kClsState]);
      float l = 0.f, o = 0.f;
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const float a = fast_ex2(s0[w * kClsState] - m);
        l = fmaf(s0[w * kClsState + 1], a, l);
        o = fmaf(s0[w * kClsState + 2 + tid], a, o);
      }
      store_any(out, out_dtype, ((int64_t)b * N * H + h) * kTcD + tid, o / l);
    }
  };
  auto stage_cls_query = [&](const Tile& x) {  // a (head, image)'s first tile: its CLS query
    if (cls_global && x.qt == 0 && tid < kTcD)
      cls_q[(x.unit & 1) * kTcD + tid] = to_f32(qg[(int64_t)x.b * qb + (int64_t)x.h * qh + tid]);
  };

  if (warp == 0) tc::tmem_alloc(tmem_slot, S::kTmemCols);
  if (tid == 0) {
    for (int i = 0; i < 5; ++i) tc::mbar_init(bar + i, 1);
    tc::fence_mbar_init();
    tma::prefetch_map(&tm_q);
    tma::prefetch_map(&tm_k);
    tma::prefetch_map(&tm_v);
    if (OTMA) tma::prefetch_map(&tm_o);
    if (t_begin < t_end) {
      const Tile x = tile_of(t_begin);
      tma::expect_tx(bar_q, kTcM * 128);
      load_rows(tc::smem_u32(sq), &tm_q, q_order, x.h, x.q0, x.b, bar_q);
      tma::expect_tx(bar_k, NB * 128);
      load_rows(tc::smem_u32(sk), &tm_k, kv_order, x.h, x.klo, x.b, bar_k);
      tma::expect_tx(bar_v, NB * 128);
      load_rows(tc::smem_u32(sv), &tm_v, kv_order, x.h, x.klo, x.b, bar_v);
    }
  }
  if (t_begin < t_end) {
    stage_bias(tile_of(t_begin), 0);
    stage_cls_query(tile_of(t_begin));
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  const uint32_t t_s = tmem, t_o = tmem + NB;
  const uint32_t lane_sel = (uint32_t)(warp * 32) << 16;
  bool ok = true;
  // the last local tile whose Q, K and V copies were issued, for the drain
  int q_last = t_begin < t_end ? 0 : -1, k_last = q_last, v_last = q_last;
  // the unit whose first tile precedes t_begin has its CLS row elsewhere
  const int first_owned_unit = (t_begin % ntq == 0) ? t_begin / ntq : t_begin / ntq + 1;

  // this warp's CLS state for the (head, image) in progress
  float cls_m = -INFINITY, cls_l = 0.f, cls_o[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  int i = 0;
  for (int t = t_begin; t < t_end && ok; ++t, ++i) {
    const Tile x = tile_of(t);
    const bool has_next = t + 1 < t_end;
    const Tile xn = tile_of(has_next ? t + 1 : t);
    const int kvalid = x.khi - x.klo;
    const int kpad = (kvalid + 31) & ~31;
    const float* sbias = sbias2 + (i & 1) * NB;
    const int qi = x.q0 + tid;
    const bool cls_tile = cls_global && x.unit >= first_owned_unit;

    if (tid == 0) {
      // S = Q K^T once this tile's Q and K have landed
      ok = tc::mbar_wait(bar_q, i & 1, err) && tc::mbar_wait(bar_k, i & 1, err);
      if (ok) {
        tc::fence_after_sync();
        const uint64_t dq = tc::sw128_desc(tc::smem_u32(sq), 16), dk = tc::sw128_desc(tc::smem_u32(sk), 16);
        const uint32_t idesc_s = tc::idesc_f16(ab_bf16, 0, kTcM, kpad);
#pragma unroll
        for (int kk = 0; kk < kTcD / 16; ++kk) tc::mma_f16_ss(t_s, dq + 2 * kk, dk + 2 * kk, idesc_s, kk > 0);
        tc::mma_commit(bar_s);
      } else if (err) {
        atomicOr(err, MN_STATUS_TC_TIMEOUT);
      }
    }
    // while S = Q K^T runs, the CLS row scores this tile's own keys
    // [q0, q0 + 128), 32 per warp
    const int cls_row0 = x.q0 + warp * 32 - x.klo;
    const int cls_nvalid = max(0, min(32, min(x.q0 + kTcM, N) - (x.q0 + warp * 32)));
    float cls_s = -INFINITY;
    if (cls_tile) {
      if (!tc::mbar_wait(bar_k, i & 1, err)) { ok = false; break; }
      const float bl2 = (BIAS && (tid & 31) < cls_nvalid) ? sbias[cls_row0 + (tid & 31)] : 0.f;
      cls_warp_score<ET, false, 1>(cls_q + (x.unit & 1) * kTcD, &cls_nvalid, sk, cls_row0, nullptr, 0, 0, 0, sl2,
                                   &bl2, &cls_s);
    }
    if (!tc::mbar_wait(bar_s, i & 1, err)) { ok = false; break; }
    tc::fence_after_sync();
    // S done: Q (and K, when no CLS fold reads it) are free for the next tile
    if (has_next) {
      if (tid == 32) {
        tma::expect_tx(bar_q, kTcM * 128);
        load_rows(tc::smem_u32(sq), &tm_q, q_order, xn.h, xn.q0, xn.b, bar_q);
      } else if (tid == 64 && !late_k) {
        tma::expect_tx(bar_k, NB * 128);
        load_rows(tc::smem_u32(sk), &tm_k, kv_order, xn.h, xn.klo, xn.b, bar_k);
      }
      q_last = i + 1;
      if (!late_k) k_last = i + 1;
      stage_bias(xn, (i + 1) & 1);
      stage_cls_query(xn);
    }
    if (cls_global && warp == 3 && t == max(t_begin, t_end - 2)) {
      // two tiles before the range ends: bring the keys that the last
      // (head, image)'s CLS row will read from global memory into L2
      const Tile xl = tile_of(t_end - 1);
      if (xl.unit >= first_owned_unit)
        for (int k0 = xl.q0 + kTcM + (tid & 31) * NB; k0 < N; k0 += 32 * NB) {
          prefetch_rows(&tm_k, kv_order, xl.h, k0, xl.b);
          prefetch_rows(&tm_v, kv_order, xl.h, k0, xl.b);
        }
    }
    // this row's legal keys relative to klo, and the warp's chunks
    int jlo = max(0, qi - window - x.klo);
    int jhi = min(kvalid, qi + window + 1 - x.klo);
    if (qi >= N) jhi = jlo;
    const bool has = jlo < jhi;
    const int wlo = (int)__reduce_min_sync(0xffffffffu, (unsigned)(has ? jlo : NB));
    const int whi = (int)__reduce_max_sync(0xffffffffu, (unsigned)(has ? jhi : 0));
    const int c_lo = min(wlo >> 5, TcChunks<NB>::kAll);
    int nch = whi > wlo ? ((whi + 31) >> 5) - c_lo : 0;
    if (nch > NCH || c_lo + nch > TcChunks<NB>::kAll) {  // cannot happen for window <= 16
      nch = max(0, min(NCH, TcChunks<NB>::kAll - c_lo));
      if (err && (tid & 31) == 0) atomicOr(err, MN_STATUS_TC_TIMEOUT);
    }
    float sc[NCH * 32];
#pragma unroll
    for (int u = 0; u < NCH; ++u)
      if (u < nch) tc::tmem_ld32_nowait(t_s + lane_sel + (c_lo + u) * 32, sc + u * 32);
    tc::tmem_ld_wait<NCH * 32>(sc);
    // logits (illegal keys -inf) and the row maximum
    float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
    for (int u = 0; u < NCH; ++u) {
      if (u >= nch) continue;
      const int cb = (c_lo + u) * 32;
      const float4* b4 = reinterpret_cast<const float4*>(sbias + cb);
#pragma unroll
      for (int i4 = 0; i4 < 8; ++i4) {
        float4 bb = make_float4(0.f, 0.f, 0.f, 0.f);
        if (BIAS) bb = b4[i4];
        const float bv[4] = {bb.x, bb.y, bb.z, bb.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int j = cb + i4 * 4 + e;
          float& v = sc[u * 32 + i4 * 4 + e];
          v = (j >= jlo && j < jhi) ? fmaf(v, sl2, bv[e]) : -INFINITY;
          mx4[e] = fmaxf(mx4[e], v);
        }
      }
    }
    const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
    const float msub = mx == -INFINITY ? 0.f : mx;
    // probabilities -> P; chunks outside the warp's range are zero
    float ls4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int u = 0; u < NCH; ++u) {
      if (u >= nch) continue;
      const int c = c_lo + u;
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        uint4 pk;
        uint32_t* w = reinterpret_cast<uint32_t*>(&pk);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float p0 = fast_ex2(sc[u * 32 + g * 8 + 2 * e] - msub);
          const float p1 = fast_ex2(sc[u * 32 + g * 8 + 2 * e + 1] - msub);
          ls4[(2 * e) & 3] += p0;
          ls4[(2 * e + 1) & 3] += p1;
          w[e] = pack2<ET>(p0, p1);
        }
        const int key8 = c * 4 + g;
        *reinterpret_cast<uint4*>(sp + (key8 >> 3) * (kTcM * 128) + tc::sw128_off(tid, key8 & 7)) = pk;
      }
    }
    // a warp whose rows all lie past the last query (the tail tile) leaves
    // its P rows alone: they feed only O rows that are never stored
    const bool live = x.q0 + warp * 32 < N;
    const int c_end = live ? (kpad + 31) >> 5 : 0;
    for (int c = 0; c < c_end; ++c) {
      if (c >= c_lo && c < c_lo + nch) continue;
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        const int key8 = c * 4 + g;
        *reinterpret_cast<uint4*>(sp + (key8 >> 3) * (kTcM * 128) + tc::sw128_off(tid, key8 & 7)) =
            make_uint4(0u, 0u, 0u, 0u);
      }
    }
    const float l_row = (ls4[0] + ls4[1]) + (ls4[2] + ls4[3]);
    tc::fence_async_smem();
    tc::fence_before_sync();
    __syncthreads();
    if (has_next && late_k) {  // every warp is past its reads of K
      if (tid == 64) {
        tma::expect_tx(bar_k, NB * 128);
        load_rows(tc::smem_u32(sk), &tm_k, kv_order, xn.h, xn.klo, xn.b, bar_k);
      }
      k_last = i + 1;
    }
    if (tid == 0) {
      tc::fence_after_sync();
      if (!tc::mbar_wait(bar_v, i & 1, err)) {
        ok = false;
        if (err) atomicOr(err, MN_STATUS_TC_TIMEOUT);
      } else {
        const uint64_t dp = tc::sw128_desc(tc::smem_u32(sp), 16);
        const uint64_t dv = tc::sw128_desc(tc::smem_u32(sv), 16384);
        const int nsteps = kpad / 16;
#pragma unroll
        for (int kk = 0; kk < NB / 16; ++kk)  // unrolled: descriptor offsets are constants
          if (kk < nsteps)
            tc::mma_f16_ss(t_o, dp + (uint64_t)((kk >> 2) * (kTcM * 128 / 16) + (kk & 3) * 2), dv + 128 * kk,
                           idesc_o, kk > 0 ? 1u : 0u);
        tc::mma_commit(bar_o);
      }
    }
    if (cls_tile) {  // while P.V runs, the CLS row folds in its scored keys
      if (!tc::mbar_wait(bar_v, i & 1, err)) { ok = false; break; }
      cls_warp_fold<ET, false, 1>(&cls_s, cls_m, cls_l, cls_o, x.qt == 0, &cls_nvalid, sv, cls_row0, nullptr, 0, 0,
                                  0);
    }
    if (!tc::mbar_wait(bar_o, i & 1, err)) { ok = false; break; }
    tc::fence_after_sync();
    // P.V done (and, after the barrier, every warp's CLS reads): V is free
    // (with the TMA store, once the stored tile has been read out of it)
    if (has_next && !OTMA) {
      if (cls_tile) __syncthreads();
      if (tid == 96) {
        tma::expect_tx(bar_v, NB * 128);
        load_rows(tc::smem_u32(sv), &tm_v, kv_order, xn.h, xn.klo, xn.b, bar_v);
      }
      v_last = i + 1;
    }
    if (OTMA) {
      // 16-bit output: the tile's O rows go to the V stage, swizzled as the
      // output map's 128-row box, and one bulk tensor store writes them
      // (rows past the sequence end are clipped); the next V copy waits
      // until the store has read the stage
      if (cls_tile) __syncthreads();  // every warp's CLS fold is done reading V
      if (live) {
        const float inv = l_row > 0.f ? 1.0f / l_row : 0.f;
#pragma unroll
        for (int c = 0; c < kTcD / 32; ++c) {
          float o[32];
          tc::tmem_ld32(t_o + lane_sel + c * 32, o);  // warp-collective: every row loads
#pragma unroll
          for (int k2 = 0; k2 < 32; ++k2) o[k2] *= inv;
#pragma unroll
          for (int k2 = 0; k2 < 4; ++k2)
            *reinterpret_cast<uint4*>(sv + tc::sw128_off(tid, c * 4 + k2)) =
                out_dtype == MN_F16 ? pack8<__half>(o + 8 * k2) : pack8<__nv_bfloat16>(o + 8 * k2);
        }
      }
      tc::fence_async_smem();
      __syncthreads();
      if (tid == 96) {
        if (o_order == 0)
          tma::store_4d(&tm_o, tc::smem_u32(sv), 0, x.h, x.q0, x.b);
        else
          tma::store_4d(&tm_o, tc::smem_u32(sv), 0, x.q0, x.h, x.b);
        tma::bulk_commit();
        tma::bulk_wait_read<0>();
        if (has_next) {  // recomputed here: xn need not stay live through the epilogue
          const Tile xv = tile_of(t + 1);
          tma::expect_tx(bar_v, NB * 128);
          load_rows(tc::smem_u32(sv), &tm_v, kv_order, xv.h, xv.klo, xv.b, bar_v);
        }
      }
      if (has_next) v_last = i + 1;
    } else {
      const float inv = l_row > 0.f ? 1.0f / l_row : 0.f;
      const int64_t obase = (((int64_t)x.b * N + qi) * H + x.h) * kTcD;
#pragma unroll
      for (int c = 0; c < kTcD / 32; ++c) {
        if (!live) break;
        float o[32];
        tc::tmem_ld32(t_o + lane_sel + c * 32, o);  // warp-collective: every row loads
        if (qi >= N) continue;
#pragma unroll
        for (int k2 = 0; k2 < 32; ++k2) o[k2] *= inv;
        if (out_dtype == MN_F32) {
          float4* dst = reinterpret_cast<float4*>(static_cast<float*>(out) + obase + c * 32);
#pragma unroll
          for (int k2 = 0; k2 < 8; ++k2)
            dst[k2] = make_float4(o[4 * k2], o[4 * k2 + 1], o[4 * k2 + 2], o[4 * k2 + 3]);
        } else if (out_dtype == MN_F16) {
          uint4* dst = reinterpret_cast<uint4*>(static_cast<__half*>(out) + obase + c * 32);
#pragma unroll
          for (int k2 = 0; k2 < 4; ++k2) dst[k2] = pack8<__half>(o + 8 * k2);
        } else {
          uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(out) + obase + c * 32);
#pragma unroll
          for (int k2 = 0; k2 < 4; ++k2) dst[k2] = pack8<__nv_bfloat16>(o + 8 * k2);
        }
      }
    }
    // the CLS row is complete after the unit's last tile
    if (cls_tile && x.qt == ntq - 1) {
      cls_warp_publish(cls_m, cls_l, cls_o, cls_st + ((x.unit & 1) * 4 + warp) * kClsState);
      if (OTMA && tid == 96) tma::bulk_wait_all();  // the windowed row 0 is written before the CLS row
      __syncthreads();  // every warp's state, and this tile's row-0 store, are in
      cls_combine(cls_st + (x.unit & 1) * 4 * kClsState, x.b, x.h);
    }
  }
  // The range ended inside an owned (head, image): the rest of its keys come
  // from global memory (outside the tile loop, where registers are free).
  const bool all_ok = __syncthreads_and(ok ? 1 : 0) != 0;
  if (all_ok && cls_global && t_begin < t_end) {
    const Tile x = tile_of(t_end - 1);
    if (x.unit >= first_owned_unit && x.qt < ntq - 1) {
      const float* qc = cls_q + (x.unit & 1) * kTcD;
      const ET* kbh = kg + (int64_t)x.b * kb + (int64_t)x.h * kh;
      const ET* vbh = vg + (int64_t)x.b * kb + (int64_t)x.h * kh;
      constexpr int G = 2;  // chunks of 128 keys per pass: G x 8 row loads in flight per lane
      for (int k0 = x.q0 + kTcM; k0 < N; k0 += G * kTcM) {
        const int key0 = k0 + warp * 32;
        const int lane = tid & 31;
        int nv[G];
        float bl2[G], sc[G];
#pragma unroll
        for (int g = 0; g < G; ++g) {
          nv[g] = max(0, min(32, N - (key0 + g * kTcM)));
          bl2[g] = 0.f;
          if (BIAS && lane < nv[g])
            bl2[g] =
                to_f32(from_f32<ET>(load_any(bias, bias_dtype, (int64_t)x.b * N + key0 + g * kTcM + lane))) * kLog2e;
        }
        cls_warp_score<ET, true, G>(qc, nv, nullptr, 0, kbh, kn, key0, kTcM, sl2, bl2, sc);
        cls_warp_fold<ET, true, G>(sc, cls_m, cls_l, cls_o, false, nv, nullptr, 0, vbh, kn, key0, kTcM);
      }
      cls_warp_publish(cls_m, cls_l, cls_o, cls_st + ((x.unit & 1) * 4 + warp) * kClsState);
      if (OTMA && tid == 96) tma::bulk_wait_all();
      __syncthreads();
      cls_combine(cls_st + (x.unit & 1) * 4 * kClsState, x.b, x.h);
    }
  }
  if (OTMA && tid == 96) tma::bulk_wait_all();
  if (tid == 0 && q_last >= 0) {
    // every bulk copy issued has landed before the CTA may exit
    tc::mbar_wait(bar_q, q_last & 1, nullptr);
    tc::mbar_wait(bar_k, k_last & 1, nullptr);
    tc::mbar_wait(bar_v, v_last & 1, nullptr);
  }
  if (!ok && tid == 0 && err) atomicOr(err, MN_STATUS_TC_TIMEOUT);
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, S::kTmemCols);
}

#ifndef MN_TC_PROMOTE128
#define MN_TC_PROMOTE128 true  // 128-byte head rows: no 256-byte L2 promotion
#endif
// 4-D tensor map (d, h, n, b) -- or (d, n, h, b) when heads are strided
// wider than tokens -- over a [B, N, H, 64] view with element strides sb, sn,
// sh; box = `rows` tokens of one head.  *order receives the dimension order.
template <typename ET>
static bool make_head_map(CUtensorMap* map, int* order, const void* ptr, int B, int N, int H, int64_t sb, int64_t sn,
                          int64_t sh, int rows) {
  const bool hn = sh <= sn;
  *order = hn ? 0 : 1;
  const cuuint64_t dims[4] = {(cuuint64_t)kTcD, (cuuint64_t)(hn ? H : N), (cuuint64_t)(hn ? N : H), (cuuint64_t)B};
  const cuuint64_t strides[3] = {(cuuint64_t)(hn ? sh : sn) * 2, (cuuint64_t)(hn ? sn : sh) * 2, (cuuint64_t)sb * 2};
  const cuuint32_t box[4] = {(cuuint32_t)kTcD, hn ? 1u : (cuuint32_t)rows, hn ? (cuuint32_t)rows : 1u, 1u};
  return tma::encode(map, std::is_same<ET, __nv_bfloat16>::value, 4, ptr, dims, strides, box, true, MN_TC_PROMOTE128);
}

template <typename ET, int NB, bool WIN>
static bool launch_tc(const void* q, int64_t qb, int64_t qn, int64_t qh, const void* k, const void* v, int64_t kb,
                      int64_t kn, int64_t kh, int B, int Nq, int Nk, int H, int window, float scale,
                      const void* bias, int bias_dtype, void* out, int out_dtype, int* err, cudaStream_t st,
                      bool cls_global, bool* cls_done) {
  CUtensorMap mq, mk, mv;
  int q_order = 0, kv_order = 0, v_order = 0;
  if (!make_head_map<ET>(&mq, &q_order, q, B, Nq, H, qb, qn, qh, kTcM) ||
      !make_head_map<ET>(&mk, &kv_order, k, B, Nk, H, kb, kn, kh, NB) ||
      !make_head_map<ET>(&mv, &v_order, v, B, Nk, H, kb, kn, kh, NB))
    return false;
  const size_t smem = TcSmem<NB>::bytes;
  auto kern = bias ? attn_tc_kernel<ET, NB, WIN, true> : attn_tc_kernel<ET, NB, WIN, false>;
  if (!ensure_smem(kern, smem)) return false;
  dim3 grid((Nq + kTcM - 1) / kTcM, H, B);
  // the CLS row rides along with query tile 0 when its scratch fits the P tile
  const bool cls = WIN && cls_global && Nq == Nk && Nk <= cls_max_keys<NB>();
  kern<<<grid, 128, smem, st>>>(mq, mk, mv, q_order, kv_order, Nq, Nk, H, window, scale, bias, bias_dtype, out,
                                out_dtype, err, cls ? 1 : 0, static_cast<const ET*>(q), qb, qh,
                                static_cast<const ET*>(k), static_cast<const ET*>(v), kb, kn, kh);
  *cls_done = cls;
  return true;
}

#ifndef MN_TC_WIN_TMA_STORE
#define MN_TC_WIN_TMA_STORE 1  // windowed, 16-bit output: one TMA store per 128-row tile
#endif
template <typename ET>
static bool launch_win_persistent(const void* q, int64_t qb, int64_t qn, int64_t qh, const void* k, const void* v,
                                  int64_t kb, int64_t kn, int64_t kh, int B, int N, int H, int window, float scale,
                                  const void* bias, int bias_dtype, void* out, int out_dtype, int* err, cudaStream_t st,
                                  bool cls_global, bool* cls_done) {
  CUtensorMap mq, mk, mv, mo;
  int q_order = 0, kv_order = 0, v_order = 0, o_order = 0;
  if (!make_head_map<ET>(&mq, &q_order, q, B, N, H, qb, qn, qh, kTcM) ||
      !make_head_map<ET>(&mk, &kv_order, k, B, N, H, kb, kn, kh, 160) ||
      !make_head_map<ET>(&mv, &v_order, v, B, N, H, kb, kn, kh, 160))
    return false;
  // 16-bit output [B, N, H, 64]: stored a 128-row tile at a time by TMA.
  // Measured at B=256 (same box): with the CLS row 221.8 against 225.3 us,
  // with a bias 203-256 against 226-266 us; without either the extra
  // epilogue barrier loses (182.5 against 176.5 us), so that case keeps the
  // per-thread row stores.
  const int64_t on = (int64_t)H * kTcD;
  const bool o_tma =
      MN_TC_WIN_TMA_STORE && (cls_global || bias != nullptr) && out_dtype != MN_F32 &&
      (reinterpret_cast<uintptr_t>(out) & 15) == 0 &&
      (out_dtype == MN_F16 ? make_head_map<__half>(&mo, &o_order, out, B, N, H, N * on, on, kTcD, kTcM)
                           : make_head_map<__nv_bfloat16>(&mo, &o_order, out, B, N, H, N * on, on, kTcD, kTcM));
  if (!o_tma) mo = mq;  // unused
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int total = ((N + kTcM - 1) / kTcM) * H * B;
  const int grid = std::max(1, std::min(total, 2 * sms));  // two CTAs per SM (TMEM, shared memory)
  const bool cls = cls_global;
  auto kern = o_tma ? (bias ? attn_win_persistent_kernel<ET, true, true> : attn_win_persistent_kernel<ET, false, true>)
                   : (bias ? attn_win_persistent_kernel<ET, true, false> : attn_win_persistent_kernel<ET, false, false>);
  constexpr uint32_t smem = TcSmem<160>::bytes + kClsBytes + 16;
  static_assert(smem <= 113 * 1024, "two CTAs per SM");
  if (!ensure_smem(kern, smem)) return false;
  kern<<<grid, 128, smem, st>>>(mq, mk, mv, mo, q_order, kv_order, o_order, N, H, B, window, scale,
                                bias, bias_dtype, out, out_dtype, err, cls ? 1 : 0, static_cast<const ET*>(q), qb, qh,
                                static_cast<const ET*>(k), static_cast<const ET*>(v), kb, kn, kh);
  *cls_done = cls;
  return true;
}

#ifndef MN_TC_WIN_PERSISTENT
#define MN_TC_WIN_PERSISTENT 1  // window <= 16 on the persistent kernel
#endif
#ifndef MN_TC_SINGLE_BAND
#define MN_TC_SINGLE_BAND 1  // windows up to 16: the tile's whole key band as one 160-key block
#endif
#ifndef MN_TC_BLOCK_KEYS
#define MN_TC_BLOCK_KEYS 64  // key block of the multi-block paths: 64 or 128
#endif

#ifndef MN_TC_FULL_WS
#define MN_TC_FULL_WS 1  // no window: the warp-specialised kernel (attention_ws.cu)
#endif
bool attention_ws(int dtype, const void* q, int64_t qb, int64_t qn, int64_t qh, const void* k, const void* v,
                  int64_t kb, int64_t kn, int64_t kh, int B, int Nq, int Nk, int H, float scale, const void* bias,
                  int bias_dtype, void* out, int out_dtype, int* err, cudaStream_t st);

template <typename ET>
static bool dispatch_tc(const void* q, int64_t qb, int64_t qn, int64_t qh, const void* k, const void* v, int64_t kb,
                        int64_t kn, int64_t kh, int B, int Nq, int Nk, int H, int window, float scale,
                        const void* bias, int bias_dtype, void* out, int out_dtype, int* err, cudaStream_t st,
                        bool cls_global, bool* cls_done) {
  constexpr int NBM = MN_TC_BLOCK_KEYS;
  if (MN_TC_SINGLE_BAND && window >= 0 && kTcM + 2 * window <= 160) {  // the whole band in one block
    if (MN_TC_WIN_PERSISTENT && Nq == Nk)
      return launch_win_persistent<ET>(q, qb, qn, qh, k, v, kb, kn, kh, B, Nq, H, window, scale, bias, bias_dtype,
                                       out, out_dtype, err, st, cls_global, cls_done);
    return launch_tc<ET, 160, true>(q, qb, qn, qh, k, v, kb, kn, kh, B, Nq, Nk, H, window, scale, bias, bias_dtype,
                                    out, out_dtype, err, st, cls_global, cls_done);
  }
  if (window >= 0)
    return launch_tc<ET, NBM, true>(q, qb, qn, qh, k, v, kb, kn, kh, B, Nq, Nk, H, window, scale, bias, bias_dtype,
                                    out, out_dtype, err, st, cls_global, cls_done);
  if (MN_TC_FULL_WS)
    return attention_ws(std::is_same<ET, __half>::value ? MN_F16 : MN_BF16, q, qb, qn, qh, k, v, kb, kn, kh, B, Nq,
                        Nk, H, scale, bias, bias_dtype, out, out_dtype, err, st);
  return launch_tc<ET, NBM, false>(q, qb, qn, qh, k, v, kb, kn, kh, B, Nq, Nk, H, window, scale, bias, bias_dtype,
                                   out, out_dtype, err, st, cls_global, cls_done);
}

// Whether the tensor-core kernels cover a call: fp16 / bf16, head_dim 64,
// 16-byte aligned rows, and (for the CLS-global row) a window the persistent
// kernel takes or few enough keys for the multi-block kernel's CLS scratch.
bool attention_tc_supported(int dtype, const void* q, int64_t qb, int64_t qn, int64_t qh, const void* k,
                            const void* v, int64_t kb, int64_t kn, int64_t kh, int Nq, int Nk, int D, int window,
                            bool cls_global) {
  if (D != kTcD || (dtype != MN_F16 && dtype != MN_BF16)) return false;
  auto aligned = [](const void* p, int64_t s1, int64_t s2, int64_t s3) {
    return (reinterpret_cast<uintptr_t>(p) % 16 == 0) && s1 % 8 == 0 && s2 % 8 == 0 && s3 % 8 == 0;
  };
  if (!aligned(q, qb, qn, qh) || !aligned(k, kb, kn, kh) || !aligned(v, kb, kn, kh)) return false;
  if (cls_global) {
    if (Nq != Nk || window < 0) return false;
    const bool band = MN_TC_SINGLE_BAND && kTcM + 2 * window <= 160;
    if (band && !MN_TC_WIN_PERSISTENT && Nk > cls_max_keys<160>()) return false;
    if (!band && Nk > cls_max_keys<MN_TC_BLOCK_KEYS>()) return false;
  }
  return true;
}

// Host-side dispatch used by mn_local_attention / mn_attention.  Returns
// false when the shape is not one the tensor-core kernel covers (nothing is
// launched then).
bool attention_tc(int dtype, const void* q, int64_t qb, int64_t qn, int64_t qh, const void* k, const void* v,
                  int64_t kb, int64_t kn, int64_t kh, int B, int Nq, int Nk, int H, int D, int window, float scale,
                  const void* bias, int bias_dtype, void* out, int out_dtype, int* err, cudaStream_t st,
                  bool cls_global, bool* cls_done) {
  *cls_done = false;
  if (!attention_tc_supported(dtype, q, qb, qn, qh, k, v, kb, kn, kh, Nq, Nk, D, window, cls_global)) return false;
  if (dtype == MN_F16)
    return dispatch_tc<__half>(q, qb, qn, qh, k, v, kb, kn, kh, B, Nq, Nk, H, window, scale, bias, bias_dtype, out,
                               out_dtype, err, st, cls_global, cls_done);
  return dispatch_tc<__nv_bfloat16>(q, qb, qn, qh, k, v, kb, kn, kh, B, Nq, Nk, H, window, scale, bias, bias_dtype,
                                    out, out_dtype, err, st, cls_global, cls_done);
}

}  // namespace mn

// ---------------------------------------------------------------------------
// Self-test of the bounded wait every tensor-core kernel here relies on: one
// CTA allocates TMEM as the kernels do, waits on an mbarrier phase that
// nothing completes, gives up after limit_ns, records MN_STATUS_TC_TIMEOUT
// and frees its TMEM -- the exit path a stuck copy or MMA would take.
// ---------------------------------------------------------------------------
namespace mn {
__global__ void __launch_bounds__(128, 1) tc_wait_selftest_kernel(int* status, unsigned long long limit_ns) {
  __shared__ uint64_t bar;
  __shared__ uint32_t tmem_slot;
  if (threadIdx.x < 32) tc::tmem_alloc(&tmem_slot, 32);
  if (threadIdx.x == 0) {
    tc::mbar_init(&bar, 1);
    tc::fence_mbar_init();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (threadIdx.x == 0 && !tc::mbar_wait(&bar, 0, nullptr, limit_ns) && status)
    atomicOr(status, MN_STATUS_TC_TIMEOUT);
  tc::fence_before_sync();
  __syncthreads();
  if (threadIdx.x < 32) tc::tmem_dealloc(tmem_slot, 32);
}
}  // namespace mn

extern "C" int mn_tc_wait_selftest(int* status, double limit_ms, void* stream) {
  if (!status || !(limit_ms >= 0.001 && limit_ms <= 1000.0)) return MN_ERR_ARG;
  cudaGetLastError();
  mn::tc_wait_selftest_kernel<<<1, 128, 0, static_cast<cudaStream_t>(stream)>>>(
      status, (unsigned long long)(limit_ms * 1e6));
  return cudaGetLastError() == cudaSuccess ? MN_OK : MN_ERR_LAUNCH;
}
