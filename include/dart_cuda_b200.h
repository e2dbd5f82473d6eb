/*
 * dart_cuda_b200 — C ABI of libmat_mul.so, a B200 (sm_100a) implementation
 * of G-Tensor's AFT-full training hot path.
 *
 * Two layers of entry points live in the same shared library:
 *
 *  1. The reference's own handle-based ABI (section "legacy"), with the same
 *     symbol names, argument order and semantics as the reference engine
 *     (native/src/engine.cu), so the reference's Dart FFI bridge
 *     (lib/core/tensor/cuda_engine.dart:316-425) and Python ctypes bridge
 *     (python/dart_cuda/core/tensor/cuda_engine.py:92-199) bind it unchanged.
 *     Handles are opaque pointers to engine-owned fp32 tensors with a grad
 *     buffer and an autograd closure; `backward(root)` runs the tape.
 *
 *  2. Batched raw-pointer entry points (prefix dc_) with explicit shapes, a
 *     dtype, a CUDA stream and an int status (0 = DC_OK).  They take device
 *     pointers, never allocate on the caller's behalf unless workspace is
 *     NULL, and never synchronise the device.
 *
 * All pointers passed to dc_ functions are device pointers unless stated.
 */
#ifndef DART_CUDA_B200_H
#define DART_CUDA_B200_H

#include <stddef.h>
#include <stdint.h>
#include <stdbool.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ status */
#define DC_OK 0
#define DC_ERR_INVALID 1       /* bad argument (shape, pointer, alignment)   */
#define DC_ERR_CUDA 2          /* a CUDA runtime/driver call failed          */
#define DC_ERR_UNSUPPORTED 3   /* valid request this build does not handle   */
#define DC_ERR_NOMEM 4         /* allocation failed or workspace too small   */
#define DC_ERR_DEVICE 5        /* a kernel reported a bounded-wait timeout   */

/* dtypes of the user-facing tensors */
#define DC_F32 0
#define DC_BF16 1

/* flags of the AFT entry points */
#define DC_AFT_CAUSAL 0x1        /* mask i > t (the reference's masked=true)   */
#define DC_AFT_ACCUMULATE 0x2    /* dQ/dK/dV/dW += instead of =                 */
#define DC_AFT_WS_VALID 0x4      /* workspace already holds this call's prep   */
#define DC_AFT_SIMT 0x8          /* CUDA-core contraction (cross-check path)   */
#define DC_AFT_COMPUTE_BF16 0x10 /* f32 tensors, bf16 tensor-core operands     */
#define DC_AFT_SAVE_STATS 0x20   /* forward keeps r and 1/den in the workspace;
                                    a WS_VALID backward reads them back instead
                                    of recomputing the forward contraction
                                    (ignored with DC_AFT_SIMT).  Costs 16 bytes
                                    of HBM traffic per element of Z; pays off
                                    from Tk of about 1024 on.  Forward and
                                    backward must pass the same flags.        */
/* The backward in two calls, so a data-parallel caller can all-reduce dW
 * while dK and dV are still being computed: a DC_AFT_BWD_NO_DKDV call writes
 * dQ and dW (dK, dV may be NULL) and leaves g and n in the workspace; a later
 * DC_AFT_BWD_DKDV call on the same workspace (with DC_AFT_WS_VALID) writes dK
 * and dV only (dZ, dQ, dW may be NULL). */
#define DC_AFT_BWD_NO_DKDV 0x40
#define DC_AFT_BWD_DKDV 0x80
/* Causal backward only: dW is written in the block-packed layout instead of
 * [Tq][ldw] — query rows in blocks of 256, block k holding its rows'
 * causal extent min(Tk8, 256(k+1)) columns (Tk8 = Tk rounded up to 8) row
 * after row; dc_aft_dw_packed_size gives its size in floats (53% of Tq*Tk at
 * T = 4096) and dc_aft_dw_unpack expands it.  For a data-parallel caller
 * that reduces dW across ranks: the upper triangle, zero on every rank, is
 * not moved.  No counterpart in the reference. */
#define DC_AFT_DW_PACKED 0x100
/* The persistent tensor-core kernels of this call leave n SMs (0..255) free,
 * e.g. for a collective running beside them on another stream. */
#define DC_AFT_SPARE_SMS(n) (((n)&0xff) << 16)

/* Message of the last failing call on this host thread ("" if none). */
const char *dc_last_error(void);

/* Synchronise `stream`, read and clear the device status word of the current
 * device.  Returns DC_OK, DC_ERR_DEVICE (some kernel since the last read
 * reported a condition; the bits are stored in *bits when non-NULL) or
 * DC_ERR_CUDA.  Bits:
 *   0x01-0x10  a bounded wait of a tensor-core kernel gave up (the kernel
 *              stopped early; its outputs are incomplete)
 *   0x20       dc_embedding_fwd saw a token id outside [0, V)
 *   0x40       dc_greedy_embed ran past the token buffer's capacity
 *   0x80       DC_STATUS_AFT_RANGE: an AFT-full call met inputs outside the
 *              range of its factorised stabilisation.  The kernels scale by
 *              the row maxima of w and the column maxima of K separately
 *              (the reference takes one joint maximum per (t, d)); when, for
 *              some (t, d), every visible term e^{w[t,i]-m_t} e^{K[i,d]-c_d}
 *              is below 2^-100 (e.g. a row's w and a column's K rising in
 *              opposite directions over a combined spread of about 70 or
 *              more), that output and its gradients are not reliable and this
 *              bit is set instead of the error passing silently. */
#define DC_STATUS_AFT_RANGE 0x80
int dc_device_status(void *stream, int *bits);

/* Library version string. */
const char *dc_version(void);

/* Kernel timing.  dc_profile_enable(1) brackets every kernel the library
 * launches with CUDA events on the launch stream (0 turns it off; both drop
 * earlier records).  dc_profile_read synchronises those events and writes, per
 * distinct kernel name, the name (64-byte slots in `names`), the summed
 * milliseconds and the launch count; it returns the number of kernels. */
int dc_profile_enable(int on);
int dc_profile_read(char *names, float *total_ms, int *counts, int max_entries);

/* Per-tile timeline of the AFT tensor-core kernels (development aid).  With
 * a device buffer of at least SMs*64*8*8 bytes, every later launch of a mode
 * whose bit is set in mode_mask (bit 0 forward, 1 backward recompute, 2 dK/dV,
 * 3 dW) writes, per CTA and local tile, 8 uint64 words: producer start, MMA
 * start, MMA done, epilogue start, epilogue done (global timer, ns), tile
 * index, K steps.  NULL turns it off. */
int dc_aft_trace(void *device_buffer, size_t bytes, int mode_mask);

/* ---------------------------------------------------------- AFT-full op
 * Z[b,t,:] = sigmoid(Q[b,t,:]) * sum_{i in S(t)} e^{K[b,i,:]+w[t,i]} V[b,i,:]
 *                               / sum_{i in S(t)} e^{K[b,i,:]+w[t,i]}
 * with S(t) = {i <= t} when DC_AFT_CAUSAL (Tq == Tk required), else all i<Tk.
 * Q, Z, dZ, dQ: [B, Tq, D]; K, V, dK, dV: [B, Tk, D]; contiguous, `dtype`.
 * w, dW: fp32, Tq rows of row stride ldw >= Tk (w[t*ldw + i]); w is shared
 * by the batch and dW is the sum over the batch.
 *
 * Replaces: aft_full_fwd (native/src/kernels/attention.cuh:6-40),
 * aft_full_bwd (native/src/engine.cu:522-590), aft_cross_fwd/bwd
 * (native/src/kernels/attention.cuh:41-128), batched over B sequences.
 */
int dc_aft_workspace_size(int B, int Tq, int Tk, int D, int dtype, int flags, size_t *bytes);

/* Operand-panel preparation of the following AFT calls in this process:
 * 0 (default) one launch, the column maxima of K combined inside CTA
 * clusters, for panels of up to 16 M elements (B * T * D), two launches
 * above; 1 always the two-launch form (row/column maxima, then the panels).
 * Both give the same panels bit for bit; the switch lets a caller or test
 * compare them.  No counterpart in the reference. */
int dc_aft_prep_mode(int two_launch);

/* Size in floats of a block-packed causal dW (DC_AFT_DW_PACKED), and its
 * expansion into dW [Tq][ldw] (zeros above each row's causal extent), on
 * `stream`.  No counterpart in the reference. */
int dc_aft_dw_packed_size(int Tq, int Tk, size_t *floats);
int dc_aft_dw_unpack(const float *packed, float *dW, int ldw, int Tq, int Tk, void *stream);

int dc_aft_fwd(const void *Q, const void *K, const void *V, const float *w, int ldw, void *Z,
               int B, int Tq, int Tk, int D, int dtype, int flags, void *workspace,
               size_t workspace_bytes, void *stream);

int dc_aft_bwd(const void *Q, const void *K, const void *V, const float *w, int ldw,
               const void *dZ, void *dQ, void *dK, void *dV, float *dW, int B, int Tq, int Tk,
               int D, int dtype, int flags, void *workspace, size_t workspace_bytes,
               void *stream);

/* The same with row strides (elements): ldi for Q, K, V, dQ, dK, dV and ldo
 * for Z, dZ, so one head's columns can be read from a fused [B*T, 3*H*D]
 * projection and written into a [B*T, H*D] head concatenation in place
 * (MultiHeadAFT, lib/core/attention/aft_multi_head_attention.dart:32-44). */
int dc_aft_fwd_strided(const void *Q, const void *K, const void *V, const float *w, int ldw,
                       void *Z, int B, int Tq, int Tk, int D, int ldi, int ldo, int dtype,
                       int flags, void *workspace, size_t workspace_bytes, void *stream);
int dc_aft_bwd_strided(const void *Q, const void *K, const void *V, const float *w, int ldw,
                       const void *dZ, void *dQ, void *dK, void *dV, float *dW, int B, int Tq,
                       int Tk, int D, int ldi, int ldo, int dtype, int flags, void *workspace,
                       size_t workspace_bytes, void *stream);

/* ------------------------------------------------- row-wise training ops
 * Affine LayerNorm over the last dim.  Replaces layernorm_fwd/bwd
 * (native/src/kernels/layernorm_embed.cuh:140-240).  x, y, dy, dx: [R, C]
 * fp32; gamma, beta, dgamma, dbeta: [C].  Backward accumulates into dx,
 * dgamma, dbeta when `accumulate` != 0 (the reference always accumulates).
 * dc_layernorm_bwd needs R*2 floats of workspace for the per-row partial
 * parameter gradients only when workspace is non-NULL; with NULL it
 * allocates stream-ordered scratch. */
int dc_layernorm_fwd(const float *x, const float *gamma, const float *beta, float *y, int R,
                     int C, float eps, void *stream);
int dc_layernorm_bwd(const float *x, const float *gamma, const float *dy, float *dx,
                     float *dgamma, float *dbeta, int R, int C, float eps, int accumulate,
                     void *stream);

/* Row-broadcast bias add out[i,j] = a[i,j] + b[j] and its backward
 * (da += dy, db += column sums).  Replaces add_row_broadcast_fwd/bwd
 * (native/src/kernels/elementwise.cuh:64-89). */
int dc_bias_fwd(const float *a, const float *b, float *out, int M, int N, void *stream);
int dc_bias_bwd(const float *dy, float *da, float *db, int M, int N, int accumulate,
                void *stream);

/* Label-smoothed cross-entropy with fused log-softmax.  Replaces
 * cross_entropy_fwd_hyper/bwd_hyper + ce_mean_reduce
 * (native/src/kernels/loss_optim.cuh:163-244, native/src/engine.cu:825-877).
 * logits [T, V] fp32, targets [T] int32 (device).  fwd writes the mean loss
 * to loss[0] (and the per-row losses to row_loss when non-NULL).  bwd
 * WRITES dlogits = (softmax - ((1-eps)1_y + eps/V)) * g / T, where g is read
 * from the device scalar grad_scale when non-NULL, else g = 1. */
int dc_ce_fwd(const float *logits, const int32_t *targets, float *loss, float *row_loss, int T,
              int V, float eps, void *stream);
int dc_ce_bwd(const float *logits, const int32_t *targets, const float *grad_scale,
              float *dlogits, int T, int V, float eps, void *stream);

/* Cross-entropy forward that allocates nothing (no counterpart in the
 * reference).  Same result as dc_ce_fwd(..., row_loss = NULL, ...), for
 * callers that cannot let the library allocate device memory during the
 * call.  The per-row losses live in a fixed array inside the library, so
 * T <= 65536; larger T returns DC_ERR_INVALID.  The array is shared by all
 * calls on a device: calls that overlap on the GPU race and must be
 * serialised by the caller (calls queued on one stream are ordered).  The
 * first call on each device resolves the array's device address and caches
 * it; make it before any stream capture.  The cached address does not
 * survive cudaDeviceReset: do not call this entry point on a device after
 * resetting it. */
int dc_ce_fwd_noalloc(const float *logits, const int32_t *targets, float *loss, int T, int V,
                      float eps, void *stream);

/* AdamW exactly as the reference applies it (step = t+1, decoupled weight
 * decay p -= lr*wd*p with wd = 0.001 in the reference).  Replaces
 * adam_kernel (native/src/kernels/loss_optim.cuh:255-298). */
int dc_adam_step(float *p, const float *g, float *m, float *v, int64_t n, int t, float lr,
                 float b1, float b2, float eps, float weight_decay, void *stream);

/* ------------------------------------------------------- dense layers
 * C[M,N] = epilogue(alpha * op(A) . op(B)) on the tensor cores (tf32
 * operands for DC_F32, bf16 for DC_BF16; fp32 accumulate, fp32 C).
 * op(A) = A stored [M,K] (lda >= K), or A^T with A stored [K,M] under
 * DC_GEMM_TRANS_A; op(B) = B stored [K,N] (ldb >= N), or B^T with B stored
 * [N,K] under DC_GEMM_TRANS_B.  A and B need 16-byte aligned bases and row
 * strides.  Epilogue, in this order: + bias[N] (DC_GEMM_BIAS); + R[M,N]
 * (ldr; or C itself under DC_GEMM_ACCUMULATE); then DC_GEMM_GELU (aux, when
 * non-NULL, receives the pre-activation; C = gelu(pre)) or DC_GEMM_GELU_BWD
 * (C = value * gelu'(aux)).  GELU is the reference's tanh form.  When the
 * output tiles leave SMs idle, K is split across CTAs: the splits of a tile
 * form a cluster that adds its partial tiles over distributed shared memory
 * (any epilogue, a fixed summation order), or, for a linear epilogue whose
 * residual is C itself (or a long K with few tiles), add into C with
 * atomics (the summation order then varies between runs).  Replaces matmul_fwd / the matmul closure
 * (native/src/engine.cu:480-507, native/src/kernels/matmul.cuh:27-131) plus
 * the bias add, GELU and residual adds of a Layer / FeedForward forward and
 * backward. */
#define DC_GEMM_TRANS_A 0x1
#define DC_GEMM_TRANS_B 0x2
#define DC_GEMM_BIAS 0x4
#define DC_GEMM_GELU 0x8
#define DC_GEMM_GELU_BWD 0x10
#define DC_GEMM_ACCUMULATE 0x20
int dc_gemm(const void *A, int lda, const void *B, int ldb, float *C, int ldc, int M, int N,
            int K, int dtype, int flags, float alpha, const float *bias, const float *R, int ldr,
            float *aux, int ldaux, void *stream);

/* dc_gemm whose epilogue ends with the decoder's cross-attention gate,
 * C = sigmoid(value) * gate[n] (gate [N], after the bias and the residual):
 * the query projection and dc_gate_fwd in one launch.  Replaces the
 * cross-attention of a decoder block against the one encoder row
 * (lib/core/transformers/aft/transformer_decoder_block.dart:63-67,
 * native/src/kernels/attention.cuh:41-128 at TEnc = 1) after its query
 * projection (matmul_tensors + add_tensor_row_broadcast).  Excludes GELU and
 * GELU_BWD. */
int dc_gemm_gate(const void *A, int lda, const void *B, int ldb, float *C, int ldc, int M, int N,
                 int K, int dtype, int flags, float alpha, const float *bias, const float *R,
                 int ldr, const float *gate, void *stream);

/* -------------------------------------------------- decoder step kernels
 * Token + position embedding of B sequences of T ids (int32, [B*T]):
 * out[b*T+t,:] = wte[idx,:] + wpe[t,:]; an id outside [0, V) gives a zero row
 * and sets bit 0x20 of the device status word.  The backward adds dx rows
 * into dwte (atomics) and the batch sums into dwpe (either may be NULL).
 * Replaces embedding_fwd/bwd (native/src/kernels/layernorm_embed.cuh:242-269)
 * and embedding_forward (native/src/engine.cu:794-822). */
int dc_embedding_fwd(const int32_t *idx, const float *wte, const float *wpe, float *out, int B,
                     int T, int D, int V, void *stream);
int dc_embedding_bwd(const int32_t *idx, const float *dx, float *dwte, float *dwpe, int B, int T,
                     int D, int V, void *stream);

/* AFT cross-attention against a single encoder row (TEnc = 1, the decoder's
 * dummy encoder, lib/core/transformers/aft/transformer_decoder_block.dart:63-67):
 * the one weight cancels, so out[m,n] = sigmoid(q[m,n]) * v0[n] exactly
 * (native/src/kernels/attention.cuh:41-128 at TEnc = 1).  The backward
 * writes dq and adds sum_m dout*sigmoid(q) into dv0; the key and the bias
 * entry get zero gradient. */
int dc_gate_fwd(const float *q, int ldq, const float *v0, float *out, int ldo, int M, int N,
                void *stream);
int dc_gate_bwd(const float *q, int ldq, const float *v0, const float *dz, int ldz, float *dq,
                int lddq, float *dv0, int M, int N, void *stream);

/* Greedy decoding of the logits at position p = *pos (a device int):
 * tokens[b*ldt + p+1] = argmax_v logits[b*ldl + v] (lowest index on ties),
 * x[b,:] = wte[token,:] + wpe[p+1,:] when x is non-NULL (the next step's
 * input), then *pos = p+1.  Past the capacity (p+1 >= ldt) nothing is
 * written and bit 0x40 of the device status word is set.  No counterpart in
 * the reference, which samples on the host after copying the logits back
 * (example/bin/shakespear4.dart:216). */
int dc_greedy_embed(const float *logits, int ldl, int B, int V, const float *wte,
                    const float *wpe, int *pos, int D, int32_t *tokens, int ldt, float *x,
                    void *stream);

/* Device-to-device copy of `rows` rows of width_bytes between pitched
 * buffers (stream-ordered). */
int dc_copy2d(void *dst, size_t dst_pitch, const void *src, size_t src_pitch, size_t width_bytes,
              size_t rows, void *stream);

/* Incremental causal AFT for one new position t = *pos (a device int, so a
 * captured step replays as the position advances) of B sequences (one layer,
 * H heads of hs channels, D = H*hs): qkv holds the position's fused
 * projection [B, 3D] (q | k | v, row stride ldq); w is head h's bias at
 * w + h*head_stride_w with row stride ldw >= Tmax; cache is the layer's k/v history
 * [Tmax][B*D/4][8] fp32 (rows < t filled, by earlier calls or
 * dc_kv_cache_fill); row t is appended by this call.  Z[b,:] (row stride ldz)
 * receives sigmoid(q) * sum_{i<=t} e^{k_i+w[t,i]} v_i / sum e^{k_i+w[t,i]}.
 * workspace: dc_aft_decode_workspace_size bytes, zero-filled once before its
 * first use (the kernel leaves it zeroed).  No counterpart in the reference,
 * which recomputes the whole context per token
 * (example/bin/shakespear4.dart:176-214). */
size_t dc_aft_decode_workspace_size(int B, int D, int Tmax);
int dc_aft_decode(const float *qkv, int ldq, const float *w, int ldw, long long head_stride_w,
                  float *cache, int B, int H, int hs, const int *pos, int Tmax, float *Z, int ldz,
                  void *workspace, size_t workspace_bytes, void *stream);
/* Fill cache rows [0, T) from a prefill's fused projection [B*T, 3D]. */
int dc_kv_cache_fill(const float *qkv, int ldq, int B, int T, int D, float *cache, void *stream);

/* ------------------------------------------------------------------ legacy
 * The reference's handle ABI (native/src/engine.cu).  Every returned handle
 * is owned by the caller and released with destroy_tensor; op outputs keep
 * their inputs alive for backward.  Calls run on the library's stream and
 * return after device work is ordered; host copies synchronise. */
void *create_tensor(int rows, int cols, float *host_data);           /* engine.cu:93  */
void destroy_tensor(void *h);                                          /* engine.cu:100 */
void get_tensor_data(void *h, float *host_out);                        /* engine.cu:123 */
void get_tensor_grad(void *h, float *host_out);                        /* engine.cu:128 */
void tensor_to_host(void *h, float *host_out);                         /* engine.cu:879 */
void set_tensor_data(void *h, float *host_in);                         /* engine.cu:936 */
void zero_grad(void *h);                                               /* engine.cu:133 */
void tensor_step(void *h, float lr);                                   /* engine.cu:138 */
void backward(void *root);                                             /* engine.cu:145 */
void *aft_forward(void *Q, void *K, void *V, void *WB, bool masked);   /* engine.cu:592 */
void *aft_cross_forward(void *Q, void *K, void *V, void *WB);          /* engine.cu:616 */
void *layernorm_forward(void *x, void *gamma, void *beta, float eps);  /* engine.cu:766 */
void *add_tensor_row_broadcast(void *a, void *b);                      /* engine.cu:352 */
void *cross_entropy_loss(void *logits, int32_t *host_targets, int32_t T, int32_t V); /* engine.cu:839 */
void adam_step(void *p, void *m, void *v, int32_t t, float lr, float b1, float b2,
               float eps);                                             /* engine.cu:887 */
void *add_tensors(void *a, void *b);                                   /* engine.cu:327 */
void *mul_tensors(void *a, void *b);                                   /* engine.cu:392 */
void *sum_tensor(void *a);                                             /* engine.cu:1141 */
void *mean_tensor(void *a);                                            /* engine.cu:1164 */

/* The rest of the reference ABI: present so the reference's loaders, which
 * bind every symbol eagerly, open this library; not on the AFT hot path. */
void *sub_tensors(void *a, void *b);                                   /* engine.cu:373  */
void *div_tensors(void *a, void *b);                                   /* engine.cu:414  */
void *add_tensor_scalar(void *a, void *scalar);                        /* engine.cu:268  */
void *sub_tensor_scalar(void *a, void *scalar);                        /* engine.cu:282  */
void *mul_tensor_scalar(void *a, void *scalar);                        /* engine.cu:296  */
void *div_tensor_scalar(void *a, void *scalar);                        /* engine.cu:311  */
void *pow_tensor(void *a, float exponent);                             /* engine.cu:424  */
void *relu_tensor(void *a);                                            /* engine.cu:434  */
void *gelu_tensor(void *a);                                            /* engine.cu:445  */
void *sigmoid_tensor(void *a);                                         /* engine.cu:460  */
void *tanh_tensor(void *a);                                            /* engine.cu:470  */
void *matmul_tensors(void *a, void *b);                                /* engine.cu:480  */
void *log_tensor(void *a);                                             /* engine.cu:510  */
void *concat_tensors_gpu(void **handles, int num_tensors);             /* engine.cu:637  */
void *concat_tensors_axis0_gpu(void **handles, int num_tensors);       /* engine.cu:686  */
void *embedding_forward(int *host_indices, void *wte, void *wpe, int T, int D); /* engine.cu:794 */
void sdg_step(void *p, void *m, void *v, int t, float lr);             /* engine.cu:907  */
void clip_gradients(void *h, float limit);                             /* engine.cu:925  */
void *slice_tensor(void *h, int start_row, int num_rows);              /* engine.cu:986  */
void *abs_tensor(void *a);                                             /* engine.cu:1023 */
void *softmax_forward(void *a);                                        /* engine.cu:1086 */
void *transpose_tensor(void *a);                                       /* engine.cu:1106 */
void compute_cost_matrix(void *pred_boxes, void *gt_boxes, void *cost); /* engine.cu:1127 */
void tensor_xavier_init(void *p, int n_in, int n_out, int seed);       /* engine.cu:1185 */
void tensor_zero_init(void *p);                                        /* engine.cu:1197 */
void *layer_norm_tensor(void *a, float eps);                           /* engine.cu:1228 */
void im2col_cuda(void *input, int channels, int height, int width, int kernel_h, int kernel_w,
                 int pad_h, int pad_w, int stride_h, int stride_w, void *output); /* engine.cu:1251 */
void col2im_cuda(float *d_col, int c, int h, int w, int k, int p, int s, float *d_im); /* engine.cu:1282 */

#ifdef __cplusplus
}
#endif
#endif /* DART_CUDA_B200_H */
