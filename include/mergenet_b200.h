/*
 * mergenet_b200.h -- C ABI of the B200 (sm_100a) DTEM spatial-routing library.
 *
 * Every entry point takes plain device pointers, explicit sizes and a
 * cudaStream_t (passed as void*), launches asynchronously on that stream and
 * returns an int status: 0 = launched, negative = argument error (nothing was
 * launched), positive = a data condition detected on the host.  Outputs and
 * workspaces are allocated by the caller; inputs are never written.  Kernels
 * report data conditions found on the device by OR-ing bits into the caller's
 * device status word (MN_STATUS_* below), which the caller reads when it
 * synchronises.  No entry point allocates device memory or synchronises.
 *
 * Tensors are dense row-major (C-contiguous) unless a stride argument says
 * otherwise.  Index tensors are int64 like the reference's torch.long tensors;
 * boolean tensors are one byte per element like torch.bool.
 *
 * Reference interfaces cited below are files of the MergeNet project.
 */
#ifndef MERGENET_B200_H
#define MERGENET_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* element types */
#define MN_F32 0
#define MN_F16 1
#define MN_BF16 2

/* host-side return codes */
#define MN_OK 0
#define MN_ERR_ARG (-1)          /* bad size, pointer or dtype                 */
#define MN_ERR_UNSUPPORTED (-2)  /* shape outside what the kernels are built for */
#define MN_ERR_WORKSPACE (-3)    /* workspace smaller than the size query says  */
#define MN_ERR_LAUNCH (-4)       /* cudaGetLastError reported a launch failure   */
#define MN_INFEASIBLE_BUDGET 1   /* fewer donor rows with a legal receiver than k */

/* device status bits (OR-ed into the caller's int) */
#define MN_STATUS_INFEASIBLE_BUDGET 1
#define MN_STATUS_DEGENERATE_RANGE 2 /* ThreTopK global max == min */
#define MN_STATUS_TOO_MANY_EDGES 4
#define MN_STATUS_TC_TIMEOUT 256     /* a bounded tensor-core wait gave up */

/* GEMM epilogues (mn_gemm_f16) */
#define MN_EPI_BIAS 0       /* fp16(acc + bias) */
#define MN_EPI_BIAS_GELU 1  /* fp16(gelu_erf(fp16(acc + bias))) */

/* Library version, for the loader's sanity check. */
int mn_version(void);

/* ------------------------------------------------------------------------
 * Geometry (host).  Replaces build_patch_spatial_adjacency +
 * adjacency_to_padded_neighbors, opentome/timm/dtem.py:50-127.
 * ------------------------------------------------------------------------ */

/* Width K of the padded [P,K] neighbour table of a grid and radius. */
int mn_neighbor_table_width(int grid_h, int grid_w, double radius, int* k_out);

/* Fill the [P,K] table (ascending patch order, index 0 / valid 0 padding). */
int mn_neighbor_table_fill(int grid_h, int grid_w, double radius, int k,
                           int64_t* indices, uint8_t* valid);

/* ------------------------------------------------------------------------
 * Fused routing for the canonical eval grouping (alternating_per_layer_fast,
 * even patch count): L merge layers of DTEMBlock._merge_train
 * (opentome/timm/dtem.py:1687-2223, called from LocalEncoder.forward,
 * opentome/models/mergenet/model.py:574-590) followed by the carrier block of
 * CLSHybridToMeModel.forward (model.py:1157-1183).
 * ------------------------------------------------------------------------ */
typedef struct mn_route_dims {
  int grid_h, grid_w;
  int num_patches;   /* P = grid_h * grid_w (even)                          */
  int half;          /* P / 2 = donors = receivers per layer                */
  int k_static;      /* K: width of the padded neighbour table              */
  int kc;            /* compact donor slots: max legal receivers of a donor */
  int kin;           /* max donors of one receiver                          */
  int radius_rows;   /* largest row offset between two neighbours           */
  int valid_rows[2]; /* donors with >= 1 legal receiver, per layer parity   */
  int stencil_dy1;   /* even-width stencil: max |dy| of donors at |dx| = 1,  */
  int stencil_dy3;   /* and at |dx| = 3 (-1 none); both -2: no stencil form  */
  int64_t table_ints;/* int32 entries of the routing table buffer           */
} mn_route_dims;

int mn_route_dims_query(int grid_h, int grid_w, double radius, mn_route_dims* dims);

/* Host-side fill of the routing table buffer (int32[table_ints]); the caller
 * copies it to the device once and passes it to every routing call.  Layout,
 * per layer parity q in {0,1} (q = layer % 2):
 *   slot_k  [half][kc]  static slot of each compact donor slot (or -1)
 *   slot_rx [half][kc]  receiver local index of that slot (or -1)
 *   rx_in   [half][kin] edge ids d*kc+c feeding each receiver, ascending
 *                       (the reference's sequential scatter order), or -1
 *   rx_off  [half][kin] stencil offset index of that edge (or -1) */
int mn_route_tables_fill(int grid_h, int grid_w, double radius,
                         const mn_route_dims* dims, int32_t* host_table);

/* Bytes of device workspace mn_route_and_gather needs. */
size_t mn_route_workspace_bytes(const mn_route_dims* dims, int batch,
                                int num_layers);

/*
 * x        [B, T, C]     tokens after the local blocks (T = 1 + P, CLS first),
 *                        MN_F32 / MN_F16 / MN_BF16 (routing math is fp32)
 * metrics  [L, B, T, Cm] metric-head outputs, any of the three dtypes
 * r_list   host int[L]   per-layer merge budget (parse_r schedule)
 * k        carriers      (T - 1 - sum(r_list) in the canonical model)
 * outputs: topk_x [B, k+1, C] (x dtype, CLS row first, carriers ordered by
 *          centre of mass), topk_size f32 [B, k+1], topk_idx int64 [B, k]
 *          (patch indices, aux["topk_patch_indices"]), size_out f32 [B, T],
 *          center_out f32 [B, T] (token_center after the last layer).
 * tau1/tau2: _tome_info tau1 (1.0) and ThreTopK temperature tau2 (30.0).
 * Ties: equal masses keep the lower patch index; equal centres keep the
 * lower patch index (the reference leaves both unspecified).
 */
int mn_route_and_gather(const mn_route_dims* dims, const int32_t* dev_table,
                        int batch, int channels, int metric_dim, int num_layers,
                        const int* r_list, int k, float tau1, float tau2,
                        const void* x, int x_dtype,
                        const void* metrics, int metric_dtype,
                        void* workspace, size_t workspace_bytes,
                        void* topk_x, float* topk_size, int64_t* topk_idx,
                        float* size_out, float* center_out,
                        int* status, void* stream);

/* ------------------------------------------------------------------------
 * Function-level drop-ins (arbitrary donor/receiver partitions).
 * ------------------------------------------------------------------------ */

/* sparse_spatial_score, opentome/timm/dtem.py:813-848 (kernel :361-433):
 * a [B,Na,C], b [B,Nb,C] (dtype), table [P,K] int64 + uint8, donor_patch
 * int64 [B,Na], receiver_patch int64 [B,Nb] sorted ascending per row.
 * Outputs scores [B,Na,K] (dtype), receiver_indices int64 [B,Na,K],
 * receiver_valid uint8 [B,Na,K]. */
int mn_sparse_spatial_score(int batch, int num_donors, int num_receivers,
                            int num_patches, int k, int channels, int dtype,
                            const void* a, const void* b,
                            const int64_t* neighbor_indices,
                            const uint8_t* neighbor_valid,
                            const int64_t* donor_patch,
                            const int64_t* receiver_patch, void* scores,
                            int64_t* receiver_indices, uint8_t* receiver_valid,
                            void* stream);

/* sparse_neighbor_dot, opentome/timm/dtem.py:680-687 (kernel :286-315). */
int mn_sparse_neighbor_dot(int batch, int num_donors, int num_receivers, int k,
                           int channels, int dtype, const void* a,
                           const void* b, const int64_t* receiver_indices,
                           const uint8_t* receiver_valid, void* scores,
                           void* stream);

/* sparse_weighted_transport, opentome/timm/dtem.py:1035-1067 (kernel
 * :436-468): out [B,Nb,C] = sum over edges (d,k) into slot s of
 * assignment[b,d,k] * values[b,d,:], accumulated per receiver in ascending
 * edge order without atomics.  Invalid edges contribute nothing. */
int mn_sparse_weighted_transport(int batch, int num_donors, int num_receivers,
                                 int k, int channels, int dtype,
                                 const void* assignment, const void* values,
                                 const int64_t* receiver_indices,
                                 const uint8_t* receiver_valid, void* out,
                                 int* status, void* stream);

/* Adjoint of the transport (the reference's backward, dtem.py:962-973):
 * grad_assignment [B,Na,K] = <values[b,d,:], grad_out[b,slot,:]>,
 * grad_values [B,Na,C] = sum_k assignment * grad_out[b,slot,:]. */
int mn_sparse_transport_adjoint(int batch, int num_donors, int num_receivers,
                                int k, int channels, int dtype,
                                const void* assignment, const void* values,
                                const int64_t* receiver_indices,
                                const uint8_t* receiver_valid,
                                const void* grad_out, void* grad_assignment,
                                void* grad_values, void* stream);

/* ThreTopK, opentome/utils/thetopk.py:4-43: x f32 [rows, n] -> y f32.
 * One global max-min range over all rows, per-row threshold.
 * workspace: mn_thre_topk_workspace_bytes(rows, n) bytes. */
size_t mn_thre_topk_workspace_bytes(int rows, int n);
int mn_thre_topk(int rows, int n, const float* x, int k, float temperature,
                 float* y, void* workspace, size_t workspace_bytes,
                 int* status, void* stream);

/* Gradient of ThreTopK with respect to x (the reference differentiates
 * opentome/utils/thetopk.py:4-43 by autograd): grad_y f32 [rows, n] ->
 * grad_x f32 [rows, n], including the path through the global range, whose
 * gradient is split evenly over tied maxima and minima.
 * workspace: mn_thre_topk_backward_workspace_bytes(rows, n) bytes. */
size_t mn_thre_topk_backward_workspace_bytes(int rows, int n);
int mn_thre_topk_backward(int rows, int n, const float* x, int k,
                          float temperature, const float* grad_y,
                          float* grad_x, void* workspace,
                          size_t workspace_bytes, int* status, void* stream);

/* The carrier block's soft-top-k training terms
 * (opentome/models/mergenet/model.py:1163-1206).
 *
 * mn_soft_topk_aux: aux f32 [B, C] = sum_i x[b, i, :] * soft_sel[b, i] /
 * max(sum_j soft_sel[b, j], 1e-6) over the n patch rows of x (element
 * strides x_batch_stride, x_row_stride; channels contiguous), the auxiliary
 * representation of model.py:1196-1198.  mn_soft_topk_aux_backward: its
 * gradients, grad_x [B, n, C] (x's dtype, contiguous) and grad_sel f32
 * [B, n]; workspace mn_soft_topk_aux_backward_workspace_bytes(B, n).
 * mn_carrier_ste_backward: the gradient that the straight-through carrier
 * weights topk_x * (1 + (w - w.detach())), w = soft_sel[b, topk_idx[b, j]]
 * (model.py:1176-1179), send to soft_sel: grad_sel f32 [B, n] is zeroed and
 * grad_sel[b, topk_idx[b, j]] = grad_out[b, j, :] . topk_x[b, j, :]; the
 * features' own gradient is grad_out itself.  An index outside [0, n) is
 * skipped and sets MN_STATUS_TOO_MANY_EDGES in *status. */
int mn_soft_topk_aux(int batch, int n, int channels, int dtype, const void* x,
                     int64_t x_batch_stride, int64_t x_row_stride,
                     const float* soft_sel, float* aux, void* stream);
size_t mn_soft_topk_aux_backward_workspace_bytes(int batch, int n);
int mn_soft_topk_aux_backward(int batch, int n, int channels, int dtype,
                              const void* x, int64_t x_batch_stride,
                              int64_t x_row_stride, const float* soft_sel,
                              const float* grad_aux, void* grad_x,
                              float* grad_sel, void* workspace,
                              size_t workspace_bytes, void* stream);
int mn_carrier_ste_backward(int batch, int k, int channels, int dtype,
                            const void* topk_x, int64_t x_batch_stride,
                            int64_t x_row_stride, const void* grad_out,
                            int64_t g_batch_stride, int64_t g_row_stride,
                            const int64_t* topk_idx, int n, float* grad_sel,
                            int* status, void* stream);

/* Soft-k-max block of DTEMBlock._select with the sparse spatial mask,
 * opentome/timm/dtem.py:1551-1580: scores f32 [B,Na,K] + allowed uint8 ->
 * assignment f32 [B,Na,K].  Returns MN_INFEASIBLE_BUDGET through the device
 * status when a batch row has fewer than k valid donor rows.  Limits:
 * num_donors <= 4096, k_slots <= 160 (MN_ERR_UNSUPPORTED beyond). */
size_t mn_dtem_select_workspace_bytes(int batch, int num_donors);
int mn_dtem_select(int batch, int num_donors, int k_slots, const float* scores,
                   const uint8_t* allowed, int k, float tau1, float tau2,
                   float* assignment, void* workspace, size_t workspace_bytes,
                   int* status, void* stream);

/* Gradient of that select block with respect to scores (the reference
 * differentiates dtem.py:1551-1580 by autograd): grad_assignment f32
 * [B,Na,K] -> grad_scores f32 [B,Na,K], through the masked row softmax, the
 * logsumexp row energies and ThreTopK over the batch (its range included);
 * the over-unity renormalisation divides by a detached total.  Masked slots
 * and rows with no allowed slot get zero.
 * workspace: mn_dtem_select_backward_workspace_bytes(batch, num_donors). */
size_t mn_dtem_select_backward_workspace_bytes(int batch, int num_donors);
int mn_dtem_select_backward(int batch, int num_donors, int k_slots,
                            const float* scores, const uint8_t* allowed, int k,
                            float tau1, float tau2,
                            const float* grad_assignment, float* grad_scores,
                            void* workspace, size_t workspace_bytes,
                            int* status, void* stream);

/* Soft-k-max select without any device allocation by the caller.  No
 * counterpart in the reference: it exists for callers that cannot allocate
 * device memory (no allocator of their own, or no cudaMalloc allowed on
 * their path).  Same inputs, outputs and results as mn_dtem_select; its
 * scratch is a fixed array inside the library (about 1.5 MB per GPU, held
 * until exit).  Limits: batch * num_donors <= 262144, batch <= 65536,
 * num_donors <= 4096 (MN_ERR_UNSUPPORTED beyond).  Calls that overlap on one
 * GPU share the scratch and race; order them on a single stream.  The first
 * call in each CUDA context (per device, and again after a device reset)
 * looks up the scratch address; make it before any stream capture. */
int mn_dtem_select_noalloc(int batch, int num_donors, int k_slots,
                           const float* scores, const uint8_t* allowed, int k,
                           float tau1, float tau2, float* assignment,
                           int* status, void* stream);

/* Transpose of the carrier gather: out [B,P,C] (dtype) gets carrier row i+1
 * of topk_x [B,k+1,C] at patch topk_idx[b,i]; other rows are zero (a patch
 * listed twice gets the later carrier; B <= 65535). */
int mn_carrier_scatter(int batch, int k, int num_patches, int channels,
                       int dtype, const void* topk_x, const int64_t* topk_idx,
                       void* out, void* stream);

/* ------------------------------------------------------------------------
 * Attention.
 * ------------------------------------------------------------------------ */

/* unbiased_local_attention / biased_local_attention,
 * opentome/timm/bias_local_attn.py:486-625 and :243-483, plus the CLS-global
 * row of LocalAttention.forward (:704-719).
 * q/k/v: element (b, n, h, d) at base + b*s_b + n*s_n + h*s_h + d (elements).
 * out  : [B, N, H, D] contiguous, dtype out_dtype.
 * bias : optional per-key additive bias [B, N] (NULL for the unbiased op),
 *        rounded to the q/k/v dtype like the reference's extra column.
 * window: |i - j| <= window; window < 0 means global attention.
 * cls_global: 1 = row 0 attends to every key (the LocalAttention CLS row).
 * scale: softmax scale (1/sqrt(D) in the reference).
 * The kernels are tcgen05 tensor-core kernels (fp32 accumulation,
 * probabilities rounded to the input type for P.V as FlashAttention does):
 * q/k/v must be fp16 or bf16 with head_dim 64 and 16-byte aligned rows
 * (strides multiples of 8 elements).  Anything else returns
 * MN_ERR_UNSUPPORTED with nothing launched; so does a CLS-global row with a
 * window above 16 over more keys than the kernel's CLS scratch holds.
 * status: optional device int; bit 8 set if a tensor-core wait timed out. */
int mn_local_attention(int batch, int tokens, int heads, int head_dim,
                       int dtype, const void* q, const void* k, const void* v,
                       int64_t s_b, int64_t s_n, int64_t s_h,
                       const void* bias, int bias_dtype, int window,
                       int cls_global, float scale, void* out, int out_dtype,
                       int* status, void* stream);

/* Attention of nq query rows over nk key rows, optionally windowed
 * (|i - j| <= window, window < 0 = every key): the recovery cross-attention
 * core of MyCrossAttention.forward (opentome/models/mergenet/model.py:173-188,
 * 393 carrier queries over the 785 pre-merge tokens).  Strides in elements;
 * out [B, nq, H, D] contiguous.  Same dtype / head_dim / alignment contract
 * as mn_local_attention (MN_ERR_UNSUPPORTED otherwise). */
int mn_attention(int batch, int nq, int nk, int heads, int head_dim, int dtype,
                 const void* q, int64_t q_sb, int64_t q_sn, int64_t q_sh,
                 const void* k, const void* v, int64_t kv_sb, int64_t kv_sn,
                 int64_t kv_sh, int window, float scale, void* out,
                 int out_dtype, int* status, void* stream);

/* LayerNorm(x + y) written in fp32 (y 16-bit of type half_dtype, optional):
 * the latent encoder's final norm over every carrier row, which fp16 / bf16
 * autocast runs in fp32 (opentome/models/mergenet/model.py:1195-1198),
 * fused with the residual add before it.  channels in {256, 384, 512, 768}. */
int mn_add_layernorm_f32(int64_t rows, int channels, const float* x, const void* y,
                         const float* gamma, const float* beta, float eps, float* out,
                         int half_dtype, void* stream);

/* Residual add + LayerNorm + fp16 cast over rows of a fp32 residual stream
 * (the norm1/norm2 inputs of the LocalBlock / latent Block forward under fp16
 * autocast, opentome/timm/bias_local_attn.py:867-868): s = x + y (y fp16,
 * optional); x_out = s (fp32, optional, may alias x); h_ln = LayerNorm(s)
 * (optional; gamma/beta fp32); h_raw = s rounded (optional).  y, h_ln and
 * h_raw are 16-bit of type half_dtype (MN_F16, or MN_BF16 for bf16
 * autocast).  channels in {256, 384, 512, 768}. */
int mn_add_layernorm(int64_t rows, int channels, const float* x, const void* y,
                     const float* gamma, const float* beta, float eps,
                     float* x_out, void* h_ln, void* h_raw, int half_dtype,
                     void* stream);

/* Patch unfold for the patch-embedding GEMM (timm PatchEmbed's stride-p
 * p x p convolution, opentome/models/mergenet/model.py:517-519):
 * images fp32 [batch, channels, height, width] ->
 * out fp16 [batch, height/p, width/p, channels, p, p].  p must be a multiple
 * of 8 and width of 4, buffers 16-byte aligned (else MN_ERR_UNSUPPORTED). */
int mn_patch_unfold(int batch, int channels, int height, int width, int patch,
                    const float* images, void* out, void* stream);

/* out[M, N] = epilogue(A[M, K] . W[N, K]^T + bias[N]) with fp16 A, W, bias
 * and out, fp32 accumulation in tensor memory (tcgen05).  It replaces the
 * fp16-autocast nn.Linear calls of the block MLP and projections (timm
 * Mlp.forward / Attention.forward as used by LocalBlock and the latent
 * blocks, opentome/timm/bias_local_attn.py:859-869).  With
 * MN_EPI_BIAS_GELU the output is GELU (exact erf form) of the fp16-rounded
 * linear output, rounded to fp16 again, as nn.GELU on the fp16 tensor gives.
 * Rows of A, W and out are K / K / N contiguous with strides lda / ldw / ldo
 * (elements); K must be a multiple of 64, N of 128, strides of 8, and all
 * pointers 16-byte aligned (else MN_ERR_UNSUPPORTED).  bias may be NULL. */
int mn_gemm_f16(int M, int N, int K, const void* a, int64_t lda, const void* w,
                int64_t ldw, const void* bias, int epilogue, void* out,
                int64_t ldo, int* status, void* stream);

/* Self-test of the bounded wait the tensor-core kernels share (no
 * counterpart in the reference): one CTA allocates tensor memory, waits on a
 * barrier phase that nothing completes, gives up after limit_ms (0.001 ..
 * 1000), ORs MN_STATUS_TC_TIMEOUT into *status and frees its tensor memory,
 * leaving the context usable.  It shows that a stuck copy or MMA ends in an
 * error status rather than a hang. */
int mn_tc_wait_selftest(int* status, double limit_ms, void* stream);

/* Split-precision GEMM for the fp32 Linear layers of the recovery
 * cross-attention (MyCrossAttention's q/k/v and out projections, which the
 * reference runs in fp32 with autocast off,
 * opentome/models/mergenet/model.py:140-145, :215-219):
 *   out[M, N] = out_scale * (A . W^T) + bias[N]
 * with the fp32 operands given as fp16 pairs, A = a_hi + a_lo (a_lo may be
 * NULL when A is exactly fp16) and W = w_hi + w_lo, each split as
 * hi = fp16(x), lo = fp16(x - hi) after an exact power-of-two scaling.
 * Three tcgen05 MMAs per K step (A_hi.W_hi + A_hi.W_lo + A_lo.W_hi)
 * accumulate in one fp32 accumulator: about 7e-7 relative error per product,
 * against 6e-8 for an fp32 FMA.  bias fp32 [N] or NULL; out fp32 or fp16
 * (out_dtype MN_F32 / MN_F16), row stride ldo.  K must be a multiple of 64,
 * N of 128, strides multiples of 8 elements and pointers 16-byte aligned
 * (else MN_ERR_UNSUPPORTED). */
int mn_gemm_f32_split(int M, int N, int K, const void* a_hi, const void* a_lo,
                      int64_t lda, const void* w_hi, const void* w_lo,
                      int64_t ldw, const float* bias, float out_scale,
                      void* out, int64_t ldo, int out_dtype, int* status,
                      void* stream);

/* fp32 LayerNorm of rows (MyCrossAttention's q_norm / kv_norm,
 * opentome/models/mergenet/model.py:133-134) written as the fp16 pair the
 * split GEMM takes: ys = LayerNorm(x) * scale (an exact power of two),
 * hi = fp16(ys), lo = fp16(ys - hi).  channels in {256, 384, 512, 768}. */
int mn_layernorm_split(int64_t rows, int channels, const float* x,
                       const float* gamma, const float* beta, float eps,
                       float scale, void* hi, void* lo, void* stream);

/* Patch embedding finish fused with the first block's LayerNorm (timm
 * PatchEmbed + VisionTransformer._pos_embed, then blocks[0].norm1, as the
 * LocalEncoder runs them under autocast,
 * opentome/models/mergenet/model.py:517-535): for image b and token t,
 * x_out[b, t] = cls + pos[0] (t == 0) or float(emb[b, t - 1]) + pos[t]
 * (fp32), h_ln[b, t] = LayerNorm(x_out[b, t]) (16-bit).  emb is the patch
 * projection [batch, tokens - 1, channels]; emb and h_ln have type
 * half_dtype (MN_F16 or MN_BF16); pos fp32 [tokens, channels]; cls fp32
 * [channels].  channels in {256, 384, 512, 768}. */
int mn_embed_layernorm(int batch, int tokens, int channels, const void* emb,
                       const float* pos, const float* cls, const float* gamma,
                       const float* beta, float eps, float* x_out, void* h_ln,
                       int half_dtype, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MERGENET_B200_H */
