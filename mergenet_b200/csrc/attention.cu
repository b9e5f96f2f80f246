// C-ABI entry points of the attention kernels: sliding-window attention over
// the flattened token sequence with an optional per-key bias and a global CLS
// row, replacing the FlashAttention calls of unbiased_local_attention /
// biased_local_attention (opentome/timm/bias_local_attn.py:486-625, :243-483)
// and the CLS-row SDPA of LocalAttention.forward (:704-719), plus the
// recovery cross-attention core (opentome/models/mergenet/model.py:173-188).
//
// There is one backend: the tcgen05 kernels of attention_tc.cu (fp16 / bf16,
// head_dim 64, fp32 accumulation).  A shape or dtype they do not cover is
// refused with MN_ERR_UNSUPPORTED before anything is launched; the Python
// layer casts fp32 q/k/v to fp16 first, as the reference does before its
// FlashAttention call (bias_local_attn.py:533-537).
#include "common.cuh"

namespace mn {

bool attention_tc_supported(int dtype, const void* q, int64_t qb, int64_t qn, int64_t qh, const void* k,
                            const void* v, int64_t kb, int64_t kn, int64_t kh, int Nq, int Nk, int D, int window,
                            bool cls_global);
bool attention_tc(int dtype, const void* q, int64_t qb, int64_t qn, int64_t qh, const void* k, const void* v,
                  int64_t kb, int64_t kn, int64_t kh, int B, int Nq, int Nk, int H, int D, int window, float scale,
                  const void* bias, int bias_dtype, void* out, int out_dtype, int* err, cudaStream_t st,
                  bool cls_global, bool* cls_done);

}  // namespace mn

using namespace mn;

extern "C" int mn_attention(int batch, int nq, int nk, int heads, int head_dim, int dtype, const void* q,
                            int64_t q_sb, int64_t q_sn, int64_t q_sh, const void* k, const void* v, int64_t kv_sb,
                            int64_t kv_sn, int64_t kv_sh, int window, float scale, void* out, int out_dtype,
                            int* status, void* stream) {
  if (batch < 0 || nq < 0 || nk <= 0 || heads <= 0 || head_dim <= 0) return MN_ERR_ARG;
  if ((int64_t)batch * nq == 0) return MN_OK;  // nothing to compute (empty tensors may have null pointers)
  if (!out) return MN_ERR_ARG;
  if (!q || !k || !v || dtype < 0 || dtype > 2 || out_dtype < 0 || out_dtype > 2) return MN_ERR_ARG;
  if (!attention_tc_supported(dtype, q, q_sb, q_sn, q_sh, k, v, kv_sb, kv_sn, kv_sh, nq, nk, head_dim, window, false))
    return MN_ERR_UNSUPPORTED;
  cudaGetLastError();
  bool cls_unused = false;
  if (!attention_tc(dtype, q, q_sb, q_sn, q_sh, k, v, kv_sb, kv_sn, kv_sh, batch, nq, nk, heads, head_dim, window,
                    scale, nullptr, 0, out, out_dtype, status, static_cast<cudaStream_t>(stream), false,
                    &cls_unused))
    return MN_ERR_UNSUPPORTED;
  return cudaGetLastError() == cudaSuccess ? MN_OK : MN_ERR_LAUNCH;
}

extern "C" int mn_local_attention(int batch, int tokens, int heads, int head_dim, int dtype, const void* q,
                                  const void* k, const void* v, int64_t s_b, int64_t s_n, int64_t s_h,
                                  const void* bias, int bias_dtype, int window, int cls_global, float scale,
                                  void* out, int out_dtype, int* status, void* stream) {
  if (batch < 0 || tokens < 0 || heads <= 0 || head_dim <= 0) return MN_ERR_ARG;
  if ((int64_t)batch * tokens == 0) return MN_OK;  // nothing to compute (empty tensors may have null pointers)
  if (!out) return MN_ERR_ARG;
  if (!q || !k || !v) return MN_ERR_ARG;
  if (dtype < 0 || dtype > 2 || out_dtype < 0 || out_dtype > 2 || (bias && (bias_dtype < 0 || bias_dtype > 2)))
    return MN_ERR_ARG;
  const bool cls_row = cls_global && window >= 0 && tokens > 1;
  if (!attention_tc_supported(dtype, q, s_b, s_n, s_h, k, v, s_b, s_n, s_h, tokens, tokens, head_dim, window,
                              cls_row))
    return MN_ERR_UNSUPPORTED;
  cudaGetLastError();
  bool cls_done = false;  // the kernel computed the CLS row itself
  if (!attention_tc(dtype, q, s_b, s_n, s_h, k, v, s_b, s_n, s_h, batch, tokens, tokens, heads, head_dim, window,
                    scale, bias, bias_dtype, out, out_dtype, status, static_cast<cudaStream_t>(stream), cls_row,
                    &cls_done) ||
      cls_row != cls_done)
    return MN_ERR_UNSUPPORTED;  // unreachable: attention_tc_supported covers the same cases
  return cudaGetLastError() == cudaSuccess ? MN_OK : MN_ERR_LAUNCH;
}
