// Persistent, warp-specialised tcgen05 GEMM for the block MLP:
//
//   out[M, N] = epilogue(A[M, K] . W[N, K]^T + bias[N])     (fp16 in, fp32 accumulate)
//
// with A the fp16 activations (rows K-contiguous) and W an nn.Linear weight
// [N, K].  The epilogues reproduce what the reference computes under fp16
// autocast: F.linear rounds its output to fp16 (bias added in fp32 first),
// and nn.GELU (exact erf form) then runs on that fp16 tensor and rounds again
// (timm Mlp.forward; opentome/timm/bias_local_attn.py:859-869).
//
// Roles (one CTA per SM, tiles handed out round-robin):
//   warp 0      TMA producer: A and W k-blocks (128B-swizzled) into a ring of
//               shared-memory stages, completion counted on mbarriers;
//   warp 1      MMA issuer: one thread issues tcgen05.mma (M=128, N=BN,
//               K=16) per 16-wide K step into one of two TMEM accumulators;
//   warps 2..9  epilogue: two warps per TMEM lane quadrant, each reading half
//               of the accumulator columns, bias (+ GELU), fp16 stores.
// The two accumulators let the epilogue of one tile overlap the main loop of
// the next.  Every wait is bounded; a timeout sets MN_STATUS_TC_TIMEOUT.
//
// Split-precision mode (mn_gemm_f32_split): the fp32 operands arrive as fp16
// pairs, x = x_hi + x_lo with x_hi = fp16(x) and x_lo = fp16(x - x_hi), the
// weight scaled by an exact power of two first so both halves stay in fp16's
// normal range.  Each 16-wide K step issues three MMAs into the same fp32
// accumulator, A_hi.W_hi + A_hi.W_lo + A_lo.W_hi (the dropped A_lo.W_lo is
// 2^-22 of a product); each operand half is exact to 2^-22 relative, so a
// product is exact to about 3 * 2^-22 (7e-7) relative, against fp32's
// 6e-8 per product and its accumulation error of a few 1e-7 over K = 384.
// With an fp16-exact A (A_lo == 0) the A_lo term is skipped.  The epilogue
// unscales, adds an fp32 bias and stores fp32 or fp16.

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "tc_common.cuh"
#include "tma.cuh"

namespace mn {
namespace gemm {

constexpr int BM = 128;
constexpr int BK = 64;  // one 128-byte swizzle atom of fp16
constexpr int kEpiWarps = 8;
constexpr int kThreads = (2 + kEpiWarps) * 32;

// Each epilogue warp stages a 32-row x 32-column block in shared memory and
// writes it with one TMA store; with fp16 output two buffers per warp let the
// next block be staged while the previous store drains.

// NA / NW: fp16 planes of A / W per stage (1 plain, 2 = hi and lo);
// OUT32: fp32 output (32 x 32 x 4-byte staging blocks, one per warp).
template <int BN, int NA = 1, int NW = 1, bool OUT32 = false>
struct Cfg {
  static constexpr uint32_t kABytes = BM * BK * 2;
  static constexpr uint32_t kBBytes = BN * BK * 2;
  static constexpr uint32_t kStageBytes = NA * kABytes + NW * kBBytes;
  static constexpr uint32_t kBlockOutBytes = 32 * 32 * (OUT32 ? 4 : 2);
  static constexpr int kOutBufs = OUT32 ? 1 : 2;
  static constexpr uint32_t kOutTotal = kEpiWarps * kOutBufs * kBlockOutBytes;
  static constexpr int kStages = std::min<int>(8, (227 * 1024 - kOutTotal - 2048) / kStageBytes);
  static constexpr int kTmemCols = 2 * BN <= 256 ? 256 : 512;  // two accumulators
  static constexpr uint32_t out_off = kStages * kStageBytes;
  static constexpr uint32_t bar_off = out_off + kOutTotal;  // full[S], empty[S], acc_full[2], acc_empty[2], done
  static constexpr uint32_t slot_off = bar_off + (2 * kStages + 5) * 8;
  static constexpr uint32_t bytes = slot_off + 16 + 1024;  // + alignment slack
};
static_assert(Cfg<256>::bytes <= 227 * 1024 && Cfg<192>::bytes <= 227 * 1024 && Cfg<128>::bytes <= 227 * 1024,
              "shared memory");
static_assert(Cfg<128, 2, 2, true>::bytes <= 227 * 1024 && Cfg<128, 2, 2, true>::kStages >= 2 &&
                  Cfg<128, 2, 2, false>::bytes <= 227 * 1024 && Cfg<128, 1, 2, true>::kStages >= 3,
              "shared memory (split precision)");

// GELU(x) = 0.5 x (1 + erf(x / sqrt 2)) on a pair, packed fp32x2.  erf(z) is
// z * P(z^2) with |z| clamped to 2.9: P of degree 9, fitted by
// mergenet_b200/csrc/gelu_fit.py (weighted least squares on Chebyshev nodes);
// max |erf error| 4.5e-5 in float32 including the clamp, so
// |GELU error| <= 2.3e-5 |x|, below half an fp16 ulp of the result for
// |x| >= 0.2 and below 5e-6 in absolute terms for smaller |x|.
constexpr float kErfClamp = 2.9f;
__device__ __forceinline__ float2 splat(float c) { return make_float2(c, c); }
__device__ __forceinline__ float2 gelu2(float2 x) {
  float2 z = fmul2(x, splat(0.70710678118654752f));
  z.x = fminf(fmaxf(z.x, -kErfClamp), kErfClamp);
  z.y = fminf(fmaxf(z.y, -kErfClamp), kErfClamp);
  const float2 u = fmul2(z, z);
  float2 p = splat(-4.687449096e-09f);
  p = ffma2(p, u, splat(2.359513331e-07f));
  p = ffma2(p, u, splat(-5.365900961e-06f));
  p = ffma2(p, u, splat(7.382134936e-05f));
  p = ffma2(p, u, splat(-6.972589181e-04f));
  p = ffma2(p, u, splat(4.874169827e-03f));
  p = ffma2(p, u, splat(-2.638702281e-02f));
  p = ffma2(p, u, splat(1.124738082e-01f));
  p = ffma2(p, u, splat(-3.760007918e-01f));
  p = ffma2(p, u, splat(1.128367066e+00f));
  const float2 e = fmul2(z, p);
  const float2 h = fmul2(x, make_float2(0.5f, 0.5f));
  return ffma2(h, e, h);
}

// EPI: 0 bias, 1 bias + GELU (fp16 bias), 2 scale * acc + fp32 bias (split).
template <int BN, int EPI, int NA = 1, int NW = 1, bool OUT32 = false>
__global__ void __launch_bounds__(kThreads, 1) gemm_tc_kernel(const __grid_constant__ CUtensorMap tmap_a,
                                                              const __grid_constant__ CUtensorMap tmap_w,
                                                              const __grid_constant__ CUtensorMap tmap_o,
                                                              const __grid_constant__ CUtensorMap tmap_a_lo,
                                                              const __grid_constant__ CUtensorMap tmap_w_lo, int M,
                                                              int N, int K, const void* __restrict__ bias_ptr,
                                                              float out_scale, int* __restrict__ err) {
  using C = Cfg<BN, NA, NW, OUT32>;
  const __half* bias = EPI == 2 ? nullptr : static_cast<const __half*>(bias_ptr);
  const float* bias32 = EPI == 2 ? static_cast<const float*>(bias_ptr) : nullptr;
  constexpr int S = C::kStages;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(base + C::bar_off);
  uint64_t* empty = full + S;
  uint64_t* acc_full = empty + S;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* done = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base + C::slot_off);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_m = (M + BM - 1) / BM, num_n = N / BN, kblocks = K / BK;
  const int tiles = num_m * num_n;

  if (warp == 1) tc::tmem_alloc(tmem_slot, C::kTmemCols);
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      tc::mbar_init(full + s, 1);
      tc::mbar_init(empty + s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(acc_full + b, 1);
      tc::mbar_init(acc_empty + b, kEpiWarps);
    }
    tc::mbar_init(done, 1);
    tc::fence_mbar_init();
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_a)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_w)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_o)) : "memory");
    if (NA == 2) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_a_lo)) : "memory");
    if (NW == 2) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_w_lo)) : "memory");
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int last_phase[8];
      for (int s = 0; s < 8; ++s) last_phase[s] = -1;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        const int mb = t / num_n, nb = t % num_n;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!tc::mbar_wait(empty + stage, phase ^ 1u, err)) { ok = false; break; }
          const uint32_t sa = tc::smem_u32(base + stage * C::kStageBytes);
          tma::expect_tx(full + stage, C::kStageBytes);
          // stage layout: A_hi [A_lo] W_hi [W_lo]
          tma::load_2d(sa, &tmap_a, kb * BK, mb * BM, full + stage);
          if (NA == 2) tma::load_2d(sa + C::kABytes, &tmap_a_lo, kb * BK, mb * BM, full + stage);
          tma::load_2d(sa + NA * C::kABytes, &tmap_w, kb * BK, nb * BN, full + stage);
          if (NW == 2) tma::load_2d(sa + NA * C::kABytes + C::kBBytes, &tmap_w_lo, kb * BK, nb * BN, full + stage);
          last_phase[stage] = (int)phase;
          if (++stage == S) { stage = 0; phase ^= 1u; }
        }
      }
      // every copy this thread issued has landed before the CTA may exit
      for (int s = 0; s < S; ++s)
        if (last_phase[s] >= 0) tc::mbar_wait(full + s, (uint32_t)last_phase[s], nullptr);
      if (!ok && err) atomicOr(err, MN_STATUS_TC_TIMEOUT);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA
    if (lane == 0) {
      constexpr uint32_t idesc = tc::idesc_f16(0, 0, BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        if (!tc::mbar_wait(acc_empty + acc, acc_phase ^ 1u, err)) { ok = false; break; }
        tc::fence_after_sync();
        const uint32_t d = tmem + acc * BN;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!tc::mbar_wait(full + stage, phase, err)) { ok = false; break; }
          tc::fence_after_sync();
          const uint32_t sa = tc::smem_u32(base + stage * C::kStageBytes);
          const uint32_t sa_lo = sa + C::kABytes;
          const uint32_t sb = sa + NA * C::kABytes;
          const uint32_t sb_lo = sb + C::kBBytes;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            tc::mma_f16_ss(d, tc::sw128_desc(sa + k * 32, 16), tc::sw128_desc(sb + k * 32, 16), idesc,
                           (kb > 0 || k > 0) ? 1u : 0u);
            if (NW == 2)
              tc::mma_f16_ss(d, tc::sw128_desc(sa + k * 32, 16), tc::sw128_desc(sb_lo + k * 32, 16), idesc, 1u);
            if (NA == 2)
              tc::mma_f16_ss(d, tc::sw128_desc(sa_lo + k * 32, 16), tc::sw128_desc(sb + k * 32, 16), idesc, 1u);
          }
          tc::mma_commit(empty + stage);  // the stage is free once these MMAs have read it
          if (++stage == S) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        tc::mma_commit(acc_full + acc);
        if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
      }
      // all MMAs issued by this thread have completed before TMEM is freed
      tc::mma_commit(done);
      tc::mbar_wait(done, 0, nullptr);
      if (!ok && err) atomicOr(err, MN_STATUS_TC_TIMEOUT);
    }
  } else {
    // ----------------------------------------------------------- epilogue
    const int ew = warp - 2;
    const int quad = warp & 3;  // TMEM lanes this warp may access
    const int col_half = ew >> 2;
    const uint32_t lane_sel = (uint32_t)(quad * 32) << 16;
    uint8_t* stage_out = base + C::out_off + ew * C::kOutBufs * C::kBlockOutBytes;
    int acc = 0, buf = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
      const int mb = t / num_n, nb = t % num_n;
      if (!tc::mbar_wait(acc_full + acc, acc_phase, err)) { ok = false; break; }
      tc::fence_after_sync();
      const __half* brow = bias ? bias + nb * BN : nullptr;
#pragma unroll 1
      for (int c = col_half * (BN / 64); c < (col_half + 1) * (BN / 64); ++c) {
        float v[32];
        tc::tmem_ld32(tmem + acc * BN + c * 32 + lane_sel, v);
        if (c == (col_half + 1) * (BN / 64) - 1) {
          // the accumulator is fully read: hand it back to the MMA warp
          tc::fence_before_sync();
          __syncwarp();
          if (lane == 0) tma::arrive(acc_empty + acc);
        }
        if (EPI == 2) {  // split precision: unscale, fp32 bias
          const float* b32 = bias32 ? bias32 + nb * BN + c * 32 : nullptr;
#pragma unroll
          for (int i = 0; i < 32; i += 4) {
            const float4 bb = b32 ? __ldg(reinterpret_cast<const float4*>(b32 + i)) : make_float4(0.f, 0.f, 0.f, 0.f);
            v[i] = fmaf(v[i], out_scale, bb.x);
            v[i + 1] = fmaf(v[i + 1], out_scale, bb.y);
            v[i + 2] = fmaf(v[i + 2], out_scale, bb.z);
            v[i + 3] = fmaf(v[i + 3], out_scale, bb.w);
          }
        }
        uint4 packed[OUT32 ? 8 : 4];
        uint32_t* pw = reinterpret_cast<uint32_t*>(packed);
        if (OUT32) {
#pragma unroll
          for (int i = 0; i < 32; ++i) pw[i] = __float_as_uint(v[i]);
        } else {
          uint4 bq[4];
          if (brow) {
            const uint4* b4 = reinterpret_cast<const uint4*>(brow + c * 32);
#pragma unroll
            for (int q = 0; q < 4; ++q) bq[q] = __ldg(b4 + q);
          }
          const __half2* bh = reinterpret_cast<const __half2*>(bq);
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            float2 p = make_float2(v[2 * i], v[2 * i + 1]);
            if (brow) p = fadd2(p, __half22float2(bh[i]));
            if (EPI == 1) p = gelu2(__half22float2(__float22half2_rn(p)));  // GELU of the fp16 linear output
            __half2 h = __float22half2_rn(p);
            pw[i] = *reinterpret_cast<uint32_t*>(&h);
          }
        }
        // stage this warp's 32 x 32 block (row = lane) and store it with TMA
        if (lane == 0) {  // the buffer's previous store has read it
          if (C::kOutBufs == 2) tma::bulk_wait_read<1>();
          else tma::bulk_wait_read<0>();
        }
        __syncwarp();
        uint8_t* sb = stage_out + buf * C::kBlockOutBytes;
        constexpr int kRowBytes = OUT32 ? 128 : 64;
#pragma unroll
        for (int q = 0; q < kRowBytes / 16; ++q) *reinterpret_cast<uint4*>(sb + lane * kRowBytes + q * 16) = packed[q];
        tc::fence_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma::store_2d(&tmap_o, tc::smem_u32(sb), nb * BN + c * 32, mb * BM + quad * 32);
          tma::bulk_commit();
        }
        if (C::kOutBufs == 2) buf ^= 1;
      }
      if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
    }
    if (lane == 0) tma::bulk_wait_all();  // stores complete before the CTA exits
    __syncwarp();
    if (!ok && lane == 0 && err) atomicOr(err, MN_STATUS_TC_TIMEOUT);
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) tc::tmem_dealloc(tmem, C::kTmemCols);
}

// ------------------------------------------------------------------ host
// 2-D fp16 tensor map over rows x cols (cols contiguous, row stride ld
// elements) with a box_rows x box_cols box; operand maps use the 128-byte
// swizzle the MMA descriptors expect, the output map a plain row-major box.
static bool make_map(CUtensorMap* map, const void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows,
                     int box_cols, bool swizzle) {
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  const cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  return tma::encode(map, false, 2, ptr, dims, strides, box, swizzle);
}

template <int BN, int EPI>
static int launch(int M, int N, int K, const void* a, int64_t lda, const void* w, int64_t ldw, const void* bias,
                  void* out, int64_t ldo, int* status, cudaStream_t st) {
  CUtensorMap ma, mw, mo;
  if (!make_map(&ma, a, M, K, lda, BM, BK, true) || !make_map(&mw, w, N, K, ldw, BN, BK, true) ||
      !make_map(&mo, out, M, N, ldo, 32, 32, false))
    return MN_ERR_UNSUPPORTED;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int tiles = ((M + BM - 1) / BM) * (N / BN);
  const int grid = std::max(1, std::min(tiles, sms));
  auto kern = gemm_tc_kernel<BN, EPI>;
  if (!ensure_smem(kern, Cfg<BN>::bytes)) return MN_ERR_LAUNCH;
  kern<<<grid, kThreads, Cfg<BN>::bytes, st>>>(ma, mw, mo, ma, mw, M, N, K, bias, 1.0f, status);
  return MN_OK;
}

// Split-precision launch: A = a_hi (+ a_lo), W = w_hi + w_lo, BN = 128.
template <int NA, bool OUT32>
static int launch_split(int M, int N, int K, const void* a_hi, const void* a_lo, int64_t lda, const void* w_hi,
                        const void* w_lo, int64_t ldw, const float* bias, float out_scale, void* out, int64_t ldo,
                        int* status, cudaStream_t st) {
  constexpr int BN = 128;
  CUtensorMap ma, mal, mw, mwl, mo;
  const cuuint64_t odims[2] = {(cuuint64_t)N, (cuuint64_t)M};
  const cuuint64_t ostr[1] = {(cuuint64_t)ldo * (OUT32 ? 4 : 2)};
  const cuuint32_t obox[2] = {32, 32};
  if (!make_map(&ma, a_hi, M, K, lda, BM, BK, true) || !make_map(&mw, w_hi, N, K, ldw, BN, BK, true) ||
      !make_map(&mwl, w_lo, N, K, ldw, BN, BK, true) ||
      (NA == 2 && !make_map(&mal, a_lo, M, K, lda, BM, BK, true)) ||
      !tma::encode_dt(&mo, OUT32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, out, odims,
                      ostr, obox, false))
    return MN_ERR_UNSUPPORTED;
  if (NA != 2) mal = ma;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int tiles = ((M + BM - 1) / BM) * (N / BN);
  const int grid = std::max(1, std::min(tiles, sms));
  using C = Cfg<BN, NA, 2, OUT32>;
  auto kern = gemm_tc_kernel<BN, 2, NA, 2, OUT32>;
  if (!ensure_smem(kern, C::bytes)) return MN_ERR_LAUNCH;
  kern<<<grid, kThreads, C::bytes, st>>>(ma, mw, mo, mal, mwl, M, N, K, bias, out_scale, status);
  return MN_OK;
}

}  // namespace gemm
}  // namespace mn

using namespace mn;

extern "C" int mn_gemm_f16(int M, int N, int K, const void* a, int64_t lda, const void* w, int64_t ldw,
                           const void* bias, int epilogue, void* out, int64_t ldo, int* status, void* stream) {
  if (M < 0 || N <= 0 || K <= 0 || !a || !w || !out) return MN_ERR_ARG;
  if (M == 0) return MN_OK;
  if (epilogue != MN_EPI_BIAS && epilogue != MN_EPI_BIAS_GELU) return MN_ERR_ARG;
  // TMA: 16-byte aligned bases and row strides; whole 64-wide k-blocks
  auto al16 = [](const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; };
  if (K % gemm::BK != 0 || lda < K || ldw < K || lda % 8 != 0 || ldw % 8 != 0 || ldo % 8 != 0 || ldo < N ||
      !al16(a) || !al16(w) || !al16(out) || (bias && !al16(bias)))
    return MN_ERR_UNSUPPORTED;
  cudaGetLastError();
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int rc = MN_ERR_UNSUPPORTED;
  const bool gelu = epilogue == MN_EPI_BIAS_GELU;
  if (N % 256 == 0)
    rc = gelu ? gemm::launch<256, 1>(M, N, K, a, lda, w, ldw, bias, out, ldo, status, st)
              : gemm::launch<256, 0>(M, N, K, a, lda, w, ldw, bias, out, ldo, status, st);
  else if (N % 192 == 0)
    rc = gelu ? gemm::launch<192, 1>(M, N, K, a, lda, w, ldw, bias, out, ldo, status, st)
              : gemm::launch<192, 0>(M, N, K, a, lda, w, ldw, bias, out, ldo, status, st);
  else if (N % 128 == 0)
    rc = gelu ? gemm::launch<128, 1>(M, N, K, a, lda, w, ldw, bias, out, ldo, status, st)
              : gemm::launch<128, 0>(M, N, K, a, lda, w, ldw, bias, out, ldo, status, st);
  if (rc != MN_OK) return rc;
  return cudaGetLastError() == cudaSuccess ? MN_OK : MN_ERR_LAUNCH;
}

extern "C" int mn_gemm_f32_split(int M, int N, int K, const void* a_hi, const void* a_lo, int64_t lda,
                                 const void* w_hi, const void* w_lo, int64_t ldw, const float* bias,
                                 float out_scale, void* out, int64_t ldo, int out_dtype, int* status, void* stream) {
  if (M < 0 || N <= 0 || K <= 0 || !a_hi || !w_hi || !w_lo || !out) return MN_ERR_ARG;
  if (out_dtype != MN_F32 && out_dtype != MN_F16) return MN_ERR_ARG;
  if (M == 0) return MN_OK;
  auto al16 = [](const void* p) { return p == nullptr || reinterpret_cast<uintptr_t>(p) % 16 == 0; };
  if (K % gemm::BK != 0 || N % 128 != 0 || lda < K || ldw < K || lda % 8 != 0 || ldw % 8 != 0 || ldo < N ||
      ldo % 8 != 0 || !al16(a_hi) || !al16(a_lo) || !al16(w_hi) || !al16(w_lo) || !al16(out) || !al16(bias))
    return MN_ERR_UNSUPPORTED;
  cudaGetLastError();
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int rc;
  if (a_lo)
    rc = out_dtype == MN_F32
             ? gemm::launch_split<2, true>(M, N, K, a_hi, a_lo, lda, w_hi, w_lo, ldw, bias, out_scale, out, ldo, status, st)
             : gemm::launch_split<2, false>(M, N, K, a_hi, a_lo, lda, w_hi, w_lo, ldw, bias, out_scale, out, ldo, status, st);
  else
    rc = out_dtype == MN_F32
             ? gemm::launch_split<1, true>(M, N, K, a_hi, nullptr, lda, w_hi, w_lo, ldw, bias, out_scale, out, ldo, status, st)
             : gemm::launch_split<1, false>(M, N, K, a_hi, nullptr, lda, w_hi, w_lo, ldw, bias, out_scale, out, ldo, status, st);
  if (rc != MN_OK) return rc;
  return cudaGetLastError() == cudaSuccess ? MN_OK : MN_ERR_LAUNCH;
}
