// Warp-specialised tensor-core attention over every key (no window), head_dim
// 64, fp16 / bf16: the latent-block attention with its per-key log(size) bias
// (opentome/models/mergenet/model.py:287-330) and the recovery
// cross-attention core (opentome/models/mergenet/model.py:173-188).
//
// One persistent CTA per SM runs two independent query streams ("slots").
// Each slot walks a contiguous range of (query tile, head, image) items:
//
//   * a load warp issues the TMA copies of Q (128 rows), K and V (64-key
//     blocks, three stages each) and stages each block's bias;
//   * an MMA warp issues the tcgen05 MMAs: S(g) = Q K(g)^T into one of three
//     TMEM S buffers, two blocks ahead, and, once the softmax has turned S(g)
//     into probabilities, O += P(g) V(g) with P read from tensor memory (no
//     shared-memory round trip for P);
//   * four softmax warps (one TMEM lane quadrant each, one query row per
//     thread) read S(g), keep the row's running maximum and sum, and write
//     P(g) as packed fp16 / bf16 pairs over the first half of S(g)'s columns.
//
// S(g+2) is issued right after P.V(g) (its buffer held P(g-1), so it waits
// for P.V(g-1) to complete), so the tensor core computes the next scores
// while the softmax warps work, and the two slots interleave on the SM's
// tensor core, special-function units and issue slots.  All hand-offs are
// mbarriers; every wait is bounded in time and gives up early once any CTA
// has recorded an error.
#include <algorithm>

#include "common.cuh"
#include "tc_common.cuh"
#include "tma.cuh"

namespace mn {
namespace ws {

constexpr int kD = 64;         // head dim
constexpr int kM = 128;        // query rows per tile
constexpr int kNB = 64;        // keys per block
constexpr int kStages = 3;     // K / V stages and TMEM S buffers per slot
constexpr int kSlots = 2;
constexpr int kThreads = 384;  // warps 0-7: softmax (slot = warp / 4); 8, 9: MMA; 10, 11: loads
constexpr uint32_t kQBytes = kM * 128;
constexpr uint32_t kKVBytes = kNB * 128;
constexpr float kLog2e = 1.4426950408889634f;
// a row maximum may grow by this much (log2 units) before O is rescaled: the
// probabilities stay below 2^8, inside fp16 / bf16 range
constexpr float kRescaleLog2 = 8.0f;

// per-slot barriers
enum : int {
  kQFull = 0,                    // [2] Q stage landed
  kKFull = 2,                    // [3] K stage landed
  kVFull = kKFull + kStages,     // [3] V stage landed
  kSFull = kVFull + kStages,     // [3] S(g) complete (+ bias of block g staged)
  kPFull = kSFull + kStages,     // [3] P(g) in TMEM (one arrival per softmax warp)
  kPVDone = kPFull + kStages,    // [3] O += P(g) V(g) complete
  kQFree = kPVDone + kStages,    // [2] last S of the item that used a Q stage complete
  kDrain = kQFree + 2,           // every MMA of the slot complete (exit)
  kBars = kDrain + 1
};

struct Layout {
  static constexpr uint32_t slot_bytes = 2 * kQBytes + 2 * kStages * kKVBytes;  // Q[2], K[3], V[3]
  static constexpr uint32_t q = 0;
  static constexpr uint32_t k = 2 * kQBytes;
  static constexpr uint32_t v = k + kStages * kKVBytes;
  static constexpr uint32_t bias = kSlots * slot_bytes;                 // [slot][stage][64] floats
  static constexpr uint32_t bars = bias + kSlots * kStages * kNB * 4;   // [slot][kBars]
  static constexpr uint32_t tmem_slot = bars + kSlots * kBars * 8;
  static constexpr uint32_t bytes = tmem_slot + 16 + 1024;              // + alignment slack
};
static_assert(Layout::bytes <= 227 * 1024, "shared memory");
static_assert(Layout::bytes > 114 * 1024, "one CTA per SM (it allocates all 512 TMEM columns)");

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

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

#ifndef MN_WS_POLY_PAIRS
#define MN_WS_POLY_PAIRS 4  // of every 16 probability pairs, this many take the FMA-pipe exp2
#endif

// 2^y for a pair of y <= 8 on the FMA pipe, so that part of the
// exponentials leave the special-function unit: y = n + f with n the nearest
// integer (added to 1.5 * 2^23, the float's low mantissa bits hold n) and
// f in [-0.5, 0.5]; 2^f is a degree-4 polynomial (relative error 2.7e-6,
// fitted by csrc/exp2_fit.py) and n is added to its exponent field.  y is
// clamped at -126, so masked keys (-inf) give 2^-126 instead of 0, which
// rounds to 0 in fp16 / bf16 and is far below the row sum.
__device__ __forceinline__ float2 ex2_poly2(float2 y) {
  y.x = fmaxf(y.x, -126.f);
  y.y = fmaxf(y.y, -126.f);
  const float2 magic = make_float2(12582912.f, 12582912.f);
  const float2 t = fadd2(y, magic);
  const float2 f = fadd2(y, fadd2(magic, make_float2(-t.x, -t.y)));  // y - n
  float2 p = ffma2(f, make_float2(9.570100344717503e-03f, 9.570100344717503e-03f),
                   make_float2(5.591786280274391e-02f, 5.591786280274391e-02f));
  p = ffma2(p, f, make_float2(2.402474433183670e-01f, 2.402474433183670e-01f));
  p = ffma2(p, f, make_float2(6.931217908859253e-01f, 6.931217908859253e-01f));
  p = ffma2(p, f, make_float2(9.999992847442627e-01f, 9.999992847442627e-01f));
  const int nx = __float_as_int(t.x) - 0x4B400000, ny = __float_as_int(t.y) - 0x4B400000;
  return make_float2(__int_as_float(__float_as_int(p.x) + (nx << 23)), __int_as_float(__float_as_int(p.y) + (ny << 23)));
}

// (d, h, n, b) tile coordinates; order 1 swaps the h and n dimensions
__device__ __forceinline__ void load_rows(uint32_t dst, const CUtensorMap* map, int order, int h, int n, int b,
                                          uint64_t* bar) {
  if (order == 0)
    tma::load_4d(dst, map, 0, h, n, b, bar);
  else
    tma::load_4d(dst, map, 0, n, h, b, bar);
}

template <typename ET>
__device__ __forceinline__ void store_row32(void* out, int out_dtype, int64_t off, const float* o) {
  if (out_dtype == MN_F32) {
    float4* dst = reinterpret_cast<float4*>(static_cast<float*>(out) + off);
#pragma unroll
    for (int i = 0; i < 8; ++i) dst[i] = make_float4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
  } else if (out_dtype == MN_F16) {
    uint4* dst = reinterpret_cast<uint4*>(static_cast<__half*>(out) + off);
#pragma unroll
    for (int i = 0; i < 4; ++i)
      dst[i] = make_uint4(pack2<__half>(o[8 * i], o[8 * i + 1]), pack2<__half>(o[8 * i + 2], o[8 * i + 3]),
                          pack2<__half>(o[8 * i + 4], o[8 * i + 5]), pack2<__half>(o[8 * i + 6], o[8 * i + 7]));
  } else {
    uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(out) + off);
#pragma unroll
    for (int i = 0; i < 4; ++i)
      dst[i] = make_uint4(pack2<__nv_bfloat16>(o[8 * i], o[8 * i + 1]), pack2<__nv_bfloat16>(o[8 * i + 2], o[8 * i + 3]),
                          pack2<__nv_bfloat16>(o[8 * i + 4], o[8 * i + 5]),
                          pack2<__nv_bfloat16>(o[8 * i + 6], o[8 * i + 7]));
  }
}

// Position in a slot's block sequence: block j of item il, whose query tile
// t of head h, image b.  Advanced one block at a time (no divisions).
struct Cursor {
  int j, il, t, h, b;
  __device__ __forceinline__ void next(int nblk, int T, int H) {
    if (++j < nblk) return;
    j = 0;
    ++il;
    if (++t < T) return;
    t = 0;
    if (++h < H) return;
    h = 0;
    ++b;
  }
};

template <typename ET, bool BIAS>
__global__ void __launch_bounds__(kThreads, 1) attn_ws_kernel(
    const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
    const __grid_constant__ CUtensorMap tm_v, int q_order, int kv_order, int Nq, int Nk, int H, int B, float scale,
    const void* __restrict__ bias, int bias_dtype, void* __restrict__ out, int out_dtype, int* __restrict__ err) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int slot = warp < 8 ? (warp >> 2) : (warp & 1);
  uint8_t* sb = base + slot * Layout::slot_bytes;
  float* bias_s = reinterpret_cast<float*>(base + Layout::bias) + slot * kStages * kNB;
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + Layout::bars) + slot * kBars;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base + Layout::tmem_slot);

  const int T = (Nq + kM - 1) / kM;  // query tiles per (image, head)
  const int nblk = (Nk + kNB - 1) / kNB;
  const int64_t total = (int64_t)T * H * B;
  const int64_t nstreams = (int64_t)kSlots * gridDim.x;
  const int64_t sid = (int64_t)blockIdx.x * kSlots + slot;
  const int64_t it0 = total * sid / nstreams;
  const int n_items = (int)(total * (sid + 1) / nstreams - it0);
  const int g_total = n_items * nblk;
  Cursor first;  // block 0 of the slot's first item
  first.j = 0;
  first.il = 0;
  first.t = (int)(it0 % T);
  first.h = (int)((it0 / T) % H);
  first.b = (int)(it0 / ((int64_t)T * H));

  if (warp == 0) tc::tmem_alloc(tmem_slot, 512);
  if (tid == 0) {
    for (int s = 0; s < kSlots; ++s) {
      uint64_t* bs = reinterpret_cast<uint64_t*>(base + Layout::bars) + s * kBars;
      for (int i = 0; i < kBars; ++i) {
        uint32_t count = 1;
        if (i >= kPFull && i < kPFull + kStages) count = 4;
        if (BIAS && i >= kSFull && i < kSFull + kStages) count = 2;  // MMA commit + bias staged
        tc::mbar_init(bs + i, count);
      }
    }
    tc::fence_mbar_init();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot + (uint32_t)slot * 256u;  // S buffers at +0, +64, +128; O at +192
  const uint32_t t_o = tmem + 3 * kNB;
  constexpr int ab_bf16 = std::is_same<ET, __nv_bfloat16>::value ? 1 : 0;
  bool ok = true;

  if (warp >= 10) {
    // ---------------------------------------------------------------- loads
    // K(g), V(g) (and Q at each item's first block) as soon as their stages
    // are free: up to three blocks ahead of the MMAs
    if (lane == 0) {
      tma::prefetch_map(&tm_q);
      tma::prefetch_map(&tm_k);
      tma::prefetch_map(&tm_v);
    }
    int q_last[2] = {-1, -1}, k_last[kStages] = {-1, -1, -1}, v_last[kStages] = {-1, -1, -1};
    Cursor c = first;
    // the block's bias, loaded one block ahead so its latency stays off the
    // copy issue path (log2 units, rounded to the operand type first; keys
    // past the end -inf)
    float pb[kNB / 32];
    auto fetch_bias = [&](const Cursor& cc) {
#pragma unroll
      for (int i = 0; i < kNB / 32; ++i) {
        const int key = cc.j * kNB + lane + 32 * i;
        pb[i] = key < Nk ? to_f32(from_f32<ET>(load_any(bias, bias_dtype, (int64_t)cc.b * Nk + key))) * kLog2e
                         : -INFINITY;
      }
    };
    if (BIAS && g_total > 0) fetch_bias(c);
    for (int g = 0; g < g_total && ok; ++g, c.next(nblk, T, H)) {
      const int st = g % kStages;
      if (c.j == 0) {
        const int qs = c.il & 1;
        if (c.il >= 2 && !(ok = tc::mbar_wait(bars + kQFree + qs, ((c.il - 2) >> 1) & 1, err))) break;
        if (lane == 0) {
          tma::expect_tx(bars + kQFull + qs, kQBytes);
          load_rows(tc::smem_u32(sb + Layout::q + qs * kQBytes), &tm_q, q_order, c.h, c.t * kM, c.b,
                    bars + kQFull + qs);
        }
        q_last[qs] = c.il;
      }
      // K stage free once S(g - 3) has completed
      if (g >= kStages && !(ok = tc::mbar_wait(bars + kSFull + st, ((g - kStages) / kStages) & 1, err))) break;
      if (lane == 0) {
        tma::expect_tx(bars + kKFull + st, kKVBytes);
        load_rows(tc::smem_u32(sb + Layout::k + st * kKVBytes), &tm_k, kv_order, c.h, c.j * kNB, c.b,
                  bars + kKFull + st);
      }
      k_last[st] = g;
      if (BIAS) {
        // the bias stage is free once the softmax of block g - 3 is done
        if (g >= kStages && !(ok = tc::mbar_wait(bars + kPFull + st, ((g - kStages) / kStages) & 1, err))) break;
#pragma unroll
        for (int i = 0; i < kNB / 32; ++i) bias_s[st * kNB + lane + 32 * i] = pb[i];
        __syncwarp();
        if (lane == 0) tma::arrive(bars + kSFull + st);  // the second arrival S(g) waits for
        if (g + 1 < g_total) {
          Cursor nx = c;
          nx.next(nblk, T, H);
          fetch_bias(nx);
        }
      }
      // V stage free once P.V(g - 3) has completed
      if (g >= kStages && !(ok = tc::mbar_wait(bars + kPVDone + st, ((g - kStages) / kStages) & 1, err))) break;
      if (lane == 0) {
        tma::expect_tx(bars + kVFull + st, kKVBytes);
        load_rows(tc::smem_u32(sb + Layout::v + st * kKVBytes), &tm_v, kv_order, c.h, c.j * kNB, c.b,
                  bars + kVFull + st);
      }
      v_last[st] = g;
    }
    if (!ok && lane == 0 && err) atomicOr(err, MN_STATUS_TC_TIMEOUT);
    if (lane == 0) {
      // every copy issued has landed before the CTA may release its shared memory
      for (int s = 0; s < 2; ++s)
        if (q_last[s] >= 0) tc::mbar_wait(bars + kQFull + s, (q_last[s] >> 1) & 1, nullptr);
      for (int s = 0; s < kStages; ++s) {
        if (k_last[s] >= 0) tc::mbar_wait(bars + kKFull + s, (k_last[s] / kStages) & 1, nullptr);
        if (v_last[s] >= 0) tc::mbar_wait(bars + kVFull + s, (v_last[s] / kStages) & 1, nullptr);
      }
    }
    __syncwarp();
  } else if (warp >= 8) {
    // ----------------------------------------------------------------- MMAs
    // S runs two blocks ahead of P.V: S(g + 2) is issued right after P.V(g),
    // so the softmax of block g + 1 finds its scores complete
    constexpr uint32_t idesc_o = tc::idesc_f16(ab_bf16, 1, kM, kD);
    Cursor cs = first, cpv = first;
    auto issue_s = [&](int g, const Cursor& c) -> bool {
      const int st = g % kStages;
      if (c.j == 0 && !tc::mbar_wait(bars + kQFull + (c.il & 1), (c.il >> 1) & 1, err)) return false;
      if (!tc::mbar_wait(bars + kKFull + st, (g / kStages) & 1, err)) return false;
      // S buffer free: P(g - 3), which it holds, consumed by P.V(g - 3)
      if (g >= kStages && !tc::mbar_wait(bars + kPVDone + st, ((g - kStages) / kStages) & 1, err)) return false;
      if (lane == 0) {
        tc::fence_after_sync();
        const int kvalid = min(kNB, Nk - c.j * kNB);
        const int kpad = (kvalid + 31) & ~31;
        const uint64_t dq = tc::sw128_desc(tc::smem_u32(sb + Layout::q + (c.il & 1) * kQBytes), 16);
        const uint64_t dk = tc::sw128_desc(tc::smem_u32(sb + Layout::k + st * kKVBytes), 16);
        const uint32_t idesc_s = tc::idesc_f16(ab_bf16, 0, kM, kpad);
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk)
          tc::mma_f16_ss(tmem + st * kNB, dq + 2 * kk, dk + 2 * kk, idesc_s, kk > 0 ? 1u : 0u);
        tc::mma_commit(bars + kSFull + st);
        if (c.j == nblk - 1) tc::mma_commit(bars + kQFree + (c.il & 1));
      }
      __syncwarp();
      return true;
    };
    auto issue_pv = [&](int g, const Cursor& c) -> bool {
      const int st = g % kStages;
      if (!tc::mbar_wait(bars + kPFull + st, (g / kStages) & 1, err)) return false;
      if (!tc::mbar_wait(bars + kVFull + st, (g / kStages) & 1, err)) return false;
      if (lane == 0) {
        tc::fence_after_sync();
        const int kvalid = min(kNB, Nk - c.j * kNB);
        const int nsteps = ((kvalid + 31) & ~31) / 16;
        // V: 16 key rows (2 KB, start field + 128) per K step; P: 8 TMEM columns per K step
        const uint64_t dv = tc::sw128_desc(tc::smem_u32(sb + Layout::v + st * kKVBytes), 16384);
#pragma unroll
        for (int kk = 0; kk < kNB / 16; ++kk)
          if (kk < nsteps)
            tc::mma_f16_ts(t_o, tmem + st * kNB + kk * 8, dv + 128 * kk, idesc_o, (c.j > 0 || kk > 0) ? 1u : 0u);
        tc::mma_commit(bars + kPVDone + st);
      }
      __syncwarp();
      return true;
    };
    for (int g = 0; g < 2 && g < g_total && ok; ++g, cs.next(nblk, T, H)) ok = issue_s(g, cs);
    for (int g = 0; g < g_total && ok; ++g) {
      ok = issue_pv(g, cpv);
      cpv.next(nblk, T, H);
      if (ok && g + 2 < g_total) {
        ok = issue_s(g + 2, cs);
        cs.next(nblk, T, H);
      }
    }
    if (!ok && lane == 0 && err) atomicOr(err, MN_STATUS_TC_TIMEOUT);
    if (lane == 0) {
      // every MMA issued has completed before the CTA may release its memory
      tc::mma_commit(bars + kDrain);
      tc::mbar_wait(bars + kDrain, 0, nullptr);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------- softmax
    const int wq = warp & 3;  // TMEM lane quadrant
    const int r = wq * 32 + lane;
    const uint32_t lane_sel = (uint32_t)(wq * 32) << 16;
    const float sl2 = scale * kLog2e;  // scores enter the softmax in log2 units
    int g = 0;
    Cursor c = first;
    for (int il = 0; il < n_items && ok; ++il, c.next(1, T, H)) {
      const int b = c.b, h = c.h, q0 = c.t * kM;
      const bool live = q0 + wq * 32 < Nq;  // warp-uniform: the tail tile's empty warps skip the math
      float m_run = -INFINITY, l_run = 0.f;
      for (int j = 0; j < nblk; ++j, ++g) {
        const int st = g % kStages;
        ok = tc::mbar_wait(bars + kSFull + st, (g / kStages) & 1, err);
        if (!ok) break;
        tc::fence_after_sync();
        if (live) {
          const int kvalid = min(kNB, Nk - j * kNB);
          const int nch = (kvalid + 31) >> 5;  // 32-column chunks the S MMA wrote: 1 or 2
          const uint32_t ts = tmem + st * kNB + lane_sel;
          float s[kNB];
          tc::tmem_ld32_nowait(ts, s);
          if (nch > 1) tc::tmem_ld32_nowait(ts + 32, s + 32);
          tc::tmem_ld_wait<kNB>(s);
          // pass 1: row maximum (log2 units)
          float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
          if (BIAS) {
            const float2 sl2v = make_float2(sl2, sl2);
            const float4* b4 = reinterpret_cast<const float4*>(bias_s + st * kNB);
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              if (u >= nch) break;
#pragma unroll
              for (int i4 = 0; i4 < 8; ++i4) {
                const float4 bb = b4[u * 8 + i4];
                float* x = s + u * 32 + i4 * 4;
                const float2 x01 = ffma2(make_float2(x[0], x[1]), sl2v, make_float2(bb.x, bb.y));
                const float2 x23 = ffma2(make_float2(x[2], x[3]), sl2v, make_float2(bb.z, bb.w));
                x[0] = x01.x; x[1] = x01.y; x[2] = x23.x; x[3] = x23.y;
                mx4[0] = fmaxf(mx4[0], x[0]);
                mx4[1] = fmaxf(mx4[1], x[1]);
                mx4[2] = fmaxf(mx4[2], x[2]);
                mx4[3] = fmaxf(mx4[3], x[3]);
              }
            }
          } else {
            if (kvalid < kNB) {  // the last block: keys past the end (zero rows) take no part
#pragma unroll
              for (int e = 0; e < kNB; ++e)
                if (e >= kvalid) s[e] = -INFINITY;
            }
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              if (u >= nch) break;
#pragma unroll
              for (int i = 0; i < 32; i += 4) {
                mx4[0] = fmaxf(mx4[0], s[u * 32 + i]);
                mx4[1] = fmaxf(mx4[1], s[u * 32 + i + 1]);
                mx4[2] = fmaxf(mx4[2], s[u * 32 + i + 2]);
                mx4[3] = fmaxf(mx4[3], s[u * 32 + i + 3]);
              }
            }
          }
          float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
          if (!BIAS) mx *= sl2;
          const float m_new = fmaxf(m_run, mx);
          const float m_use = (m_run == -INFINITY || m_new - m_run > kRescaleLog2) ? m_new : m_run;
          const float corr = (m_run == -INFINITY || m_use == m_run) ? 1.f : ex2(m_run - m_use);
          const float msub = m_use == -INFINITY ? 0.f : m_use;
          // pass 2: probabilities, packed in pairs over the first half of the S columns
          float2 sum2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
          const float2 nm = make_float2(-msub, -msub);
          const float2 sl2v = make_float2(sl2, sl2);
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            if (u >= nch) break;
            uint32_t pk[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const float2 x = make_float2(s[u * 32 + 2 * i], s[u * 32 + 2 * i + 1]);
              const float2 y = BIAS ? fadd2(x, nm) : ffma2(x, sl2v, nm);
              // pairs spread evenly over the row take the polynomial
              const float2 p = (MN_WS_POLY_PAIRS > 0 && (i * MN_WS_POLY_PAIRS) % 16 >= 16 - MN_WS_POLY_PAIRS)
                                   ? ex2_poly2(y)
                                   : make_float2(ex2(y.x), ex2(y.y));
              sum2[i & 1] = fadd2(sum2[i & 1], p);
              pk[i] = pack2<ET>(p.x, p.y);
            }
            tc::tmem_st16_nowait(ts + u * 16, pk);
          }
          tc::tmem_wait_st();
          // rescale the running output rows once P.V(g - 1) has completed
          // (warp-collective TMEM access: the whole warp takes part)
          if (j > 0 && __any_sync(0xffffffffu, corr != 1.f)) {
            const int gp = g - 1;
            ok = tc::mbar_wait(bars + kPVDone + gp % kStages, (gp / kStages) & 1, err);
            if (ok) {
              tc::fence_after_sync();
              float o[32];
#pragma unroll
              for (int c = 0; c < kD / 32; ++c) {
                tc::tmem_ld32(t_o + lane_sel + c * 32, o);
#pragma unroll
                for (int i = 0; i < 32; ++i) o[i] *= corr;
                tc::tmem_st32(t_o + lane_sel + c * 32, o);
              }
            }
          }
          const float2 ss = fadd2(sum2[0], sum2[1]);
          l_run = l_run * corr + (ss.x + ss.y);
          m_run = m_use;
        }
        if (!ok) break;
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) tma::arrive(bars + kPFull + st);
      }
      if (!ok) break;
      if (nblk == 0) continue;
      // epilogue: O / l once the item's last P.V has completed
      const int gl = g - 1;
      ok = tc::mbar_wait(bars + kPVDone + gl % kStages, (gl / kStages) & 1, err);
      if (!ok) break;
      tc::fence_after_sync();
      if (live) {
        const int qi = q0 + r;
        const float inv = l_run > 0.f ? 1.0f / l_run : 0.f;
        const int64_t obase = (((int64_t)b * Nq + qi) * H + h) * kD;
#pragma unroll
        for (int c = 0; c < kD / 32; ++c) {
          float o[32];
          tc::tmem_ld32(t_o + lane_sel + c * 32, o);  // warp-collective: every row loads
          if (qi >= Nq) continue;
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] *= inv;
          store_row32<ET>(out, out_dtype, obase + c * 32, o);
        }
      }
    }
    if (!ok && lane == 0 && err) atomicOr(err, MN_STATUS_TC_TIMEOUT);
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    tc::fence_after_sync();
    tc::tmem_dealloc(*tmem_slot, 512);
  }
}

}  // namespace ws

template <typename ET>
static bool make_head_map_ws(CUtensorMap* map, int* order, const void* ptr, int B, int N, int H, int64_t sb,
                             int64_t sn, int64_t sh, int rows) {
  const bool hn = sh <= sn;
  *order = hn ? 0 : 1;
  const cuuint64_t dims[4] = {(cuuint64_t)ws::kD, (cuuint64_t)(hn ? H : N), (cuuint64_t)(hn ? N : H), (cuuint64_t)B};
  const cuuint64_t strides[3] = {(cuuint64_t)(hn ? sh : sn) * 2, (cuuint64_t)(hn ? sn : sh) * 2, (cuuint64_t)sb * 2};
  const cuuint32_t box[4] = {(cuuint32_t)ws::kD, hn ? 1u : (cuuint32_t)rows, hn ? (cuuint32_t)rows : 1u, 1u};
  return tma::encode(map, std::is_same<ET, __nv_bfloat16>::value, 4, ptr, dims, strides, box, true, true);
}

// Host launch of the warp-specialised kernel (window < 0).  Returns false
// when nothing could be launched.
template <typename ET>
static bool launch_ws_t(const void* q, int64_t qb, int64_t qn, int64_t qh, const void* k, const void* v, int64_t kb,
                        int64_t kn, int64_t kh, int B, int Nq, int Nk, int H, float scale, const void* bias,
                        int bias_dtype, void* out, int out_dtype, int* err, cudaStream_t st) {
  CUtensorMap mq, mk, mv;
  int q_order = 0, kv_order = 0, v_order = 0;
  if (!make_head_map_ws<ET>(&mq, &q_order, q, B, Nq, H, qb, qn, qh, ws::kM) ||
      !make_head_map_ws<ET>(&mk, &kv_order, k, B, Nk, H, kb, kn, kh, ws::kNB) ||
      !make_head_map_ws<ET>(&mv, &v_order, v, B, Nk, H, kb, kn, kh, ws::kNB))
    return false;
  const int64_t total = (int64_t)((Nq + ws::kM - 1) / ws::kM) * H * B;
  if (total <= 0 || Nk <= 0) return true;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((total + 1) / 2, sms));
  auto kern = bias ? ws::attn_ws_kernel<ET, true> : ws::attn_ws_kernel<ET, false>;
  if (!ensure_smem(kern, ws::Layout::bytes)) return false;
  kern<<<grid, ws::kThreads, ws::Layout::bytes, st>>>(mq, mk, mv, q_order, kv_order, Nq, Nk, H, B, scale, bias,
                                                      bias_dtype, out, out_dtype, err);
  return true;
}

bool attention_ws(int dtype, const void* q, int64_t qb, int64_t qn, int64_t qh, const void* k, const void* v,
                  int64_t kb, int64_t kn, int64_t kh, int B, int Nq, int Nk, int H, float scale, const void* bias,
                  int bias_dtype, void* out, int out_dtype, int* err, cudaStream_t st) {
  if (dtype == MN_F16)
    return launch_ws_t<__half>(q, qb, qn, qh, k, v, kb, kn, kh, B, Nq, Nk, H, scale, bias, bias_dtype, out,
                               out_dtype, err, st);
  return launch_ws_t<__nv_bfloat16>(q, qb, qn, qh, k, v, kb, kn, kh, B, Nq, Nk, H, scale, bias, bias_dtype, out,
                                    out_dtype, err, st);
}

}  // namespace mn
