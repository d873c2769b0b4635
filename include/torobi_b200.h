/*
 * torobi_b200 -- C ABI of the B200 (sm_100a) backend for Torobi's
 * quantized-weight QLoRA path.
 *
 * The reference engine (takahashim/torobi, Rust) reaches its device through
 * mlx-c, whose convention this ABI keeps (docs/vendoring.md:291-297): every
 * call returns an int status (0 = ok), borrows its inputs, writes into
 * caller-owned outputs, and takes the stream it runs on.  Nothing here
 * allocates device memory in the hot calls; all buffers are the caller's.
 *
 * Data types on this boundary
 *   bf16      16-bit brain float, passed as raw device pointers
 *   codes     uint32, 32/bits codes per word packed low bits first along the
 *             last axis of the [rows, cols] weight (MLX affine layout)
 *   scales,
 *   biases    bf16 [rows, cols / group_size]; w = scale * q + bias
 *   f32       float (LoRA master parameters, gradients, optimizer moments)
 * Every device pointer must be 16-byte aligned; row pitches are the dense
 * row widths given.
 *
 * Streams are cudaStream_t passed as void* (NULL = legacy default stream).
 */
#ifndef TOROBI_B200_H
#define TOROBI_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TQ_OK 0
#define TQ_ERR_INVALID 1     /* a shape or argument the op does not accept   */
#define TQ_ERR_UNSUPPORTED 2 /* bits / group_size / rank outside the set     */
#define TQ_ERR_MISALIGNED 3  /* a pointer or row pitch breaks 16-byte rule  */
#define TQ_ERR_TIMEOUT 4     /* a device-side wait ran out (see tq_device_status) */
#define TQ_ERR_CUDA 5        /* a CUDA runtime call failed                   */
#define TQ_ERR_NCCL 6        /* an NCCL call failed                          */

#define TQ_DTYPE_F32 0
#define TQ_DTYPE_BF16 1

/* Library version (major * 10000 + minor * 100 + patch). */
int tq_version(void);

/*
 * Message of the last failing call on this host thread ("" if none).
 * Replaces the message mlx-c hands to the installed error handler
 * (engine/src/mlxc/error.rs:1-80).
 */
const char* tq_last_error(void);

/*
 * Reads (and with clear != 0 resets) the device status word of the current
 * device: bit 1 = a kernel's bounded wait ran out.  Synchronizes the device.
 * Returns TQ_OK, or TQ_ERR_TIMEOUT when the word is non-zero.
 */
int tq_device_status(int* status_out, int clear);

/*
 * Test hook for the failure path: launches one bounded wait on an mbarrier
 * that nothing arrives on.  After limit_ns (1 ms to 10 s) the wait runs out,
 * sets the timeout bit (1) of the device status word and the kernel returns,
 * as every kernel's bounded waits do when a producer is lost;
 * tq_device_status then reports TQ_ERR_TIMEOUT.  No counterpart in the
 * reference, whose engine surfaces MLX's errors instead
 * (engine/src/mlxc/error.rs:1-80).
 */
int tq_wait_selftest(int64_t limit_ns, void* stream);

/* ---------------------------------------------------------------- packing */

/*
 * MLX affine quantization of a bf16 matrix w [rows, cols] along cols:
 * codes [rows, cols*bits/32] u32, scales/biases [rows, cols/group_size] bf16.
 * bits in {4, 8}; group_size in {32, 64, 128}; cols % group_size == 0.
 * Replaces mlx_quantize (MLX 0.32.2), which the reference never binds
 * (engine/src/mlxc/ops.rs:91-130 has no quantize); it runs where imported
 * weights are converted to their declared dtype (engine/src/plan.rs:499).
 */
int tq_quantize(const void* w, int64_t rows, int64_t cols, int group_size, int bits, void* codes,
                void* scales, void* biases, void* stream);

/*
 * Inverse of tq_quantize: w [rows, cols] bf16 = RNE(scale * q + bias).
 * Replaces mlx_dequantize (MLX 0.32.2; unbound in the reference).
 */
int tq_dequantize(const void* codes, const void* scales, const void* biases, int64_t rows,
                  int64_t cols, int group_size, int bits, void* w, void* stream);

/*
 * Many matrices in one launch (every linear of a model at load time): job i
 * is tq_quantize's / tq_dequantize's arguments for one matrix, with one
 * group_size and bits for all.  Every job is checked before anything is
 * launched (errors name the job); empty jobs are skipped; more than 256
 * non-empty jobs take one launch per 256.  No counterpart in the reference
 * (quantize is not bound there); the batched form of the two above.
 */
typedef struct {
  const void* w; /* bf16 [rows, cols] */
  int64_t rows, cols;
  void* codes;   /* u32 [rows, cols * bits / 32] */
  void* scales;  /* bf16 [rows, cols / group_size] */
  void* biases;  /* bf16 [rows, cols / group_size] */
} TqQuantizeJob;

typedef struct {
  const void* codes;
  const void* scales;
  const void* biases;
  int64_t rows, cols;
  void* w; /* bf16 [rows, cols] out */
} TqDequantizeJob;

int tq_quantize_batch(const TqQuantizeJob* jobs, int n_jobs, int group_size, int bits,
                      void* stream);
int tq_dequantize_batch(const TqDequantizeJob* jobs, int n_jobs, int group_size, int bits,
                        void* stream);

/* ----------------------------------------------------------- the GEMM ---- */

/*
 * quantized_matmul with MLX's argument meaning, W the quantized
 * [w_rows, w_cols] matrix packed along w_cols:
 *   transpose != 0:  y[m, w_rows] = x[m, w_cols] . W^T   (linear forward)
 *   transpose == 0:  y[m, w_cols] = x[m, w_rows] . W     (its VJP wrt x)
 * bf16 in, f32 accumulation on the tensor cores, bf16 out.
 * Requires w_rows % 8 == 0 and w_cols % group_size == 0.
 * Replaces Op::Matmul -> mlx_matmul (engine/src/interp.rs:270,
 * engine/src/mlxc/ops.rs:108) for the frozen base weight of a linear
 * (lib/torobi/dsl/layers.rb:22), and the matmul VJP MLX derives for it
 * (engine/src/executor.rs:163-191).
 */
int tq_quantized_matmul(const void* x, const void* codes, const void* scales, const void* biases,
                        int64_t m, int64_t w_rows, int64_t w_cols, int transpose, int group_size,
                        int bits, void* y, void* stream);

/*
 * The adapted linear in one kernel: quantized_matmul (as above) plus an
 * optional bias and the LoRA up-projection accumulated into the same
 * tensor-memory accumulator before the single rounding to bf16:
 *   transpose != 0:  y = x . W^T + bias + lora_down . lora_up^T
 *                    lora_up = LoRA B [w_rows, rank]
 *   transpose == 0:  y = x . W + lora_down . lora_up
 *                    lora_up = LoRA A [rank, w_cols]   (bias must be NULL)
 * lora_down is the caller's [m, rank] bf16 down-projection, already scaled
 * by alpha/rank (tq_lora_down), with row pitch ld_down elements (0 = rank;
 * otherwise a multiple of 8 >= rank): the columns of one adapter inside the
 * stacked down-projection of linears that share x.  rank in {8, 16};
 * lora_up/lora_down NULL (rank 0) leaves the plain GEMM.
 * Replaces the node chain matmul, add, matmul, matmul, mul_scalar, add of
 * lib/torobi/dsl/layers.rb:22-24 and lib/torobi/lora.rb:79-85, dispatched at
 * engine/src/interp.rs:192,198,247,270.
 */
int tq_qlora_matmul(const void* x, const void* codes, const void* scales, const void* biases,
                    int64_t m, int64_t w_rows, int64_t w_cols, int transpose, int group_size,
                    int bits, const void* bias, const void* lora_up, const void* lora_down,
                    int64_t ld_down, int64_t rank, void* y, void* stream);

/*
 * Split-K forms of the two GEMM entry points.  When the output tiles alone
 * cannot occupy every SM (small m), the reduction is split across CTAs that
 * write f32 partials into the caller's workspace; a second kernel sums them,
 * adds the bias and rounds to bf16.  tq_qmm_workspace_bytes reports how many
 * bytes a call of this shape needs (0: it will not split); a NULL workspace
 * (or one too small) is refused when a split is planned.  The results equal
 * the plain entry points' to f32 summation order.  No reference counterpart:
 * the same replacement of mlx_matmul as tq_quantized_matmul, scheduled for
 * small token counts.
 */
int tq_qmm_workspace_bytes(int64_t m, int64_t w_rows, int64_t w_cols, int transpose,
                           int group_size, int bits, size_t* bytes);
int tq_quantized_matmul_ws(const void* x, const void* codes, const void* scales,
                           const void* biases, int64_t m, int64_t w_rows, int64_t w_cols,
                           int transpose, int group_size, int bits, void* y, void* workspace,
                           size_t workspace_bytes, void* stream);
int tq_qlora_matmul_ws(const void* x, const void* codes, const void* scales, const void* biases,
                       int64_t m, int64_t w_rows, int64_t w_cols, int transpose, int group_size,
                       int bits, const void* bias, const void* lora_up, const void* lora_down,
                       int64_t ld_down, int64_t rank, void* y, void* workspace,
                       size_t workspace_bytes, void* stream);

/*
 * tq_qlora_matmul_ws that adds its result into y instead of storing it:
 *   y = RNE(RNE(result) + y)
 * result being what tq_qlora_matmul_ws would write (bias and LoRA included),
 * so a sum of several GEMMs built by calling this in turn equals the one a
 * caller gets by adding their bf16 outputs one after another.  Used for the
 * input gradient of linears that read one x (q/k/v, gate/up): MLX's VJP sums
 * their cotangents for x (engine/src/executor.rs:163-191); this sums them in
 * the GEMM's epilogue with no separate add.  The 4-bit small-token forward
 * kernel is never used by this entry point.
 */
int tq_qlora_matmul_accumulate(const void* x, const void* codes, const void* scales,
                               const void* biases, int64_t m, int64_t w_rows, int64_t w_cols,
                               int transpose, int group_size, int bits, const void* bias,
                               const void* lora_up, const void* lora_down, int64_t ld_down,
                               int64_t rank, void* y, void* workspace, size_t workspace_bytes,
                               void* stream);

/*
 * tq_quantized_matmul with no workspace argument and no allocation: the
 * split-K partials live in a fixed 8 MiB array inside the library
 * (TQ_NOALLOC_SCRATCH_BYTES; every GPU that loads the library holds it until
 * the process exits).  For callers that cannot call cudaMalloc at call time:
 * a runtime with no device allocator of its own, or one whose device memory
 * is owned by a pool that this code may not draw from.
 * - A shape whose split needs more than the array (tq_qmm_workspace_bytes >
 *   TQ_NOALLOC_SCRATCH_BYTES) is refused with TQ_ERR_INVALID; on a 148-SM
 *   B200 every call of up to 200 tokens fits (256 tokens x 1152 outputs
 *   needs 9 MiB).
 * - The first call on a device looks up the array's device address (once per
 *   device, with that device current); make that first call before any
 *   stream capture.
 * - All calls on a device share the one array.  Nothing in it has to start
 *   at zero (each call writes every partial it reads), but calls that
 *   overlap on the GPU (different streams, no ordering between them) race.
 * Results equal tq_quantized_matmul_ws's.  No counterpart in the reference.
 */
#define TQ_NOALLOC_SCRATCH_BYTES (8u << 20)
int tq_quantized_matmul_noalloc(const void* x, const void* codes, const void* scales,
                                const void* biases, int64_t m, int64_t w_rows, int64_t w_cols,
                                int transpose, int group_size, int bits, void* y, void* stream);

/* ------------------------------------------------------- LoRA side branch */

/*
 * Down-projection of the LoRA branch, scaled, on the tensor cores:
 *   out  [m, rank] bf16 = RNE(scale * x . a^T)
 *   out_t[rank, ld_t] bf16 = the same values transposed (optional, may be
 *         NULL); ld_t >= m and ld_t % 8 == 0, columns m.. are left untouched
 * x bf16 [m, k]; a bf16 [rank, k]; f32 accumulation; rank in {8, 16}.
 * Forward: a = LoRA A, the `matmul(x, a.transpose)` of lib/torobi/lora.rb:83
 * with the `* scale` of :84 folded in.  Backward: x = dY and a = B^T, the
 * `dY . B . scale` partner of the same VJP (engine/src/executor.rs:163-191).
 * out feeds tq_qlora_matmul; out_t feeds tq_lora_grad.
 */
int tq_lora_down(const void* x, const void* a, int64_t m, int64_t k, int64_t rank, float scale,
                 void* out, void* out_t, int64_t ld_t, void* stream);

/*
 * LoRA weight gradient on the tensor cores, reduced over the m rows:
 *   out_layout == 0: g[c, rank] = sum_m x[m, c] * p_t[rank, m]   (dB = dY^T . t)
 *   out_layout == 1: g[rank, c] = sum_m p_t[rank, m] * x[m, c]   (dA = u^T . x)
 * x bf16 [m, c] (c % 8 == 0); p_t bf16 [rank, ld_p] (tq_lora_down's out_t,
 * ld_p >= m, ld_p % 8 == 0); g f32.
 * accumulate != 0 adds into g (micro-batch accumulation,
 * engine/src/state.rs:418-449); otherwise g is overwritten.
 * Replaces the matmul VJPs MLX derives for lib/torobi/lora.rb:83-84
 * (engine/src/executor.rs:163-191).
 */
int tq_lora_grad(const void* x, const void* p_t, int64_t ld_p, int64_t m, int64_t c,
                 int64_t rank, int out_layout, int accumulate, void* g, void* stream);

/* ---------------------------------------------------------- optimizer ---- */

/*
 * Sum of squares of n f32 values into *out (device f32); accumulate != 0 adds
 * to *out.  Building block of the global norm of engine/src/optimizer.rs:64-82.
 */
int tq_sumsq(const float* x, int64_t n, float* out, int accumulate, void* stream);

/*
 * One fused AdamW update over n f32 parameters, following
 * engine/src/optimizer.rs:305-352: moments, bias correction from step t
 * (the count after this step), then decoupled weight decay.
 * The gradient is read as grad * grad_scale (e.g. 1/world_size).
 * norm_sq (optional, device): sum of squares of the unscaled gradient buffer.
 *   If it is not finite the update is skipped and params/moments are left as
 *   they were (engine/src/state.rs:360-370).  If clip > 0 and
 *   sqrt(norm_sq) * |grad_scale| > clip, the gradient is further scaled by
 *   clip / that norm (engine/src/state.rs:373-376).
 * params_bf16 (optional) receives RNE(params) after the update.
 */
int tq_adamw(float* params, const float* grads, float* m, float* v, int64_t n, int64_t t,
             float lr, float beta1, float beta2, float eps, float weight_decay, float grad_scale,
             const float* norm_sq, float clip, void* params_bf16, void* stream);

/*
 * dst[cols, rows] bf16 = RNE(src[rows, cols]) transposed: the K-major copy of
 * LoRA B that the backward down-projection (tq_lora_down with a = B^T) reads.
 */
int tq_transpose_to_bf16(const float* src, int64_t rows, int64_t cols, void* dst, void* stream);

/* -------------------------------------------------------- decoder glue --- */
/*
 * The decoder operations around the quantized linears, fused (bf16 in and
 * out, f32 arithmetic).  Not part of the quantized-weight path itself; they
 * replace the reference's composed ops for the Llama-shaped block.
 *
 * RMSNorm over the last axis (engine/src/interp.rs:312-319):
 *   y = x * rsqrt(mean(x^2) + eps) * w; rstd (optional, f32 [rows]) keeps
 *   rsqrt(mean(x^2) + eps) for the backward.  hidden % 8 == 0.
 */
int tq_rmsnorm_fwd(const void* x, const void* w, int64_t rows, int64_t hidden, float eps, void* y,
                   float* rstd, void* stream);

/*
 * The pre-norm block's residual add and the norm after it in one pass:
 *   s = RNE_bf16(x + res)  (the residual stream, written to s)
 *   y = RMSNorm(s) * w     (of the stored s; rstd as above)
 * Replaces Op::Add (engine/src/interp.rs:198) followed by the RMSNorm
 * above; its backward is tq_rmsnorm_bwd on s with dres = the gradient of s.
 * There is no in-place form: s and y must not overlap x, res or each other
 * (refused with TQ_ERR_INVALID).
 */
int tq_add_rmsnorm_fwd(const void* x, const void* res, const void* w, int64_t rows,
                       int64_t hidden, float eps, void* s, void* y, float* rstd, void* stream);

/*
 * The RMSNorm's input gradient (the gain is frozen in QLoRA, so no dw):
 *   dx = rstd * dy * w - x * rstd^3 * mean(dy * w * x)  (+ dres, if not NULL).
 */
int tq_rmsnorm_bwd(const void* x, const void* w, const float* rstd, const void* dy,
                   const void* dres, int64_t rows, int64_t hidden, void* dx, void* stream);

/*
 * Rotary embedding in place or out of place on x [tokens, heads, dim] bf16
 * (tokens = batch * seq, position = token % seq): the first half of each head
 * rotates against the second, by the angles whose cos/sin are [seq, dim/2]
 * f32 (engine/src/interp.rs:350-388).  inverse != 0 rotates back (the VJP).
 */
int tq_rope(const void* x, int64_t tokens, int64_t heads, int64_t dim, int64_t seq,
            const float* cos_table, const float* sin_table, int inverse, void* y, void* stream);

/*
 * SwiGLU (lib/torobi/models/llama.rb:320-327): a = g * sigmoid(g) * u over n
 * elements, and its VJP dg, du.  n % 8 == 0.
 */
int tq_swiglu_fwd(const void* g, const void* u, int64_t n, void* a, void* stream);
int tq_swiglu_bwd(const void* g, const void* u, const void* da, int64_t n, void* dg, void* du,
                  void* stream);

/* ------------------------------------------------------------ attention --- */

/*
 * Scaled dot-product attention with grouped-query heads, the decoder's
 * attention node (engine/src/interp.rs:405-432: MLX's fused SDPA with a
 * causal mode and no mask tensor; lib/torobi/models/llama.rb:297-316):
 *   o[b, i, h, :] = sum_j softmax_j(scale * q[b, i, h, :] . k[b, j, g, :]) v[b, j, g, :]
 * with g = h / (heads / kv_heads) and, when causal != 0, j <= i only.
 * q, o [batch, seq, heads, head_dim]; k, v [batch, seq, kv_heads, head_dim];
 * bf16, contiguous (the projections' [tokens, features] output viewed per
 * head).  head_dim 64 or 128; heads a multiple of kv_heads.  lse
 * [batch, heads, seq] f32 receives each query row's natural-log
 * log-sum-exp of its scaled scores (what the backward reads).
 */
int tq_attention_fwd(const void* q, const void* k, const void* v, int64_t batch, int64_t seq,
                     int64_t heads, int64_t kv_heads, int64_t head_dim, float scale, int causal,
                     void* out, float* lse, void* stream);

/*
 * Its VJP: dq, dk, dv (the layouts of q, k, v) from the upstream gradient
 * dout and the forward's out and lse, for the same shape, scale and mode
 * (MLX differentiates its fused SDPA for the reference,
 * engine/src/executor.rs:163-191).  dk and dv sum over the query heads that
 * share a key/value head; no atomics, so the result is deterministic.
 * workspace: tq_attention_bwd_workspace_bytes() bytes of device memory,
 * 256-byte aligned (two f32 statistics per query row).
 */
int tq_attention_bwd_workspace_bytes(int64_t batch, int64_t seq, int64_t heads, size_t* bytes);
int tq_attention_bwd(const void* q, const void* k, const void* v, const void* out,
                     const void* dout, const float* lse, int64_t batch, int64_t seq,
                     int64_t heads, int64_t kv_heads, int64_t head_dim, float scale, int causal,
                     void* dq, void* dk, void* dv, void* workspace, size_t workspace_bytes,
                     void* stream);

/* --------------------------------------------------------------- export --- */

/*
 * A quantized linear merged with its LoRA pair, for export:
 *   out[r, c] = deq(r, c) + scale * sum_i lora_b[r, i] * lora_a[i, c]
 * deq = RNE_bf16(scale_g * q + bias_g) as the GEMM uses it; the low-rank sum
 * in f32, i ascending, each product and sum rounded on its own, then scaled
 * and added (so a CPU restatement matches bit for bit).  lora_a f32
 * [rank, cols], lora_b f32 [rows, rank]; rank 0 with both NULL
 * gives the dequantized weight.  out [rows, cols] f32 (out_dtype
 * TQ_DTYPE_F32) or bf16 (TQ_DTYPE_BF16, rounded once).  The merge the
 * reference's export asks for and does not have (lib/torobi/export.rb:118-140;
 * its export writes f32, engine/src/export.rs:1-9).
 */
int tq_lora_merge(const void* codes, const void* scales, const void* biases, int64_t rows,
                  int64_t cols, int group_size, int bits, const float* lora_a,
                  const float* lora_b, int64_t rank, float scale, void* out, int out_dtype,
                  void* stream);

/* ----------------------------------------------------------------- loss --- */

/*
 * Cross-entropy per position, in f32, of bf16 logits [rows, vocab] (row
 * pitch ld elements, ld >= vocab) against int64 targets [rows]:
 *   lse[r]  = log(sum_j exp(z[r, j]))       (largest logit taken out first)
 *   loss[r] = lse[r] - z[r, targets[r]]
 * No reduction: which positions count, and how, is the caller's (as the
 * reference's node: engine/src/interp.rs:434-444, config/ops.yml:212-220).
 * A target outside [0, vocab) picks nothing (loss = lse).
 */
int tq_cross_entropy_fwd(const void* logits, const int64_t* targets, int64_t rows, int64_t vocab,
                         int64_t ld, float* lse, float* loss, void* stream);

/*
 * Its VJP: dlogits[r, j] = RNE_bf16(scale * dloss[r] * (exp(z[r, j] - lse[r])
 * - [j == targets[r]])), dlogits with row pitch ld; dloss may be NULL (all
 * ones).  dlogits may be the logits buffer itself (each logit is read before
 * its gradient overwrites it), so the backward needs no second
 * [rows, vocab] buffer.
 */
int tq_cross_entropy_bwd(const void* logits, const int64_t* targets, const float* lse,
                         int64_t rows, int64_t vocab, int64_t ld, const float* dloss, float scale,
                         void* dlogits, void* stream);

/* ------------------------------------------------------ data parallel ---- */
/*
 * NCCL communicator for the data-parallel step (no reference counterpart:
 * distribution is a non-goal there, docs/plan.md:108).  The unique id is
 * 128 opaque bytes made on rank 0 and shared by the caller.
 */
int tq_dp_unique_id(void* id128);
int tq_dp_comm_init(void** comm, const void* id128, int nranks, int rank);
int tq_dp_allreduce_sum(void* comm, void* buf, int64_t count, int dtype, void* stream);
int tq_dp_comm_destroy(void* comm);
/*
 * Ends a communicator without waiting for its peers, for use after a rank
 * has been lost (its collectives may never complete, so a destroy could
 * wait for good).  The reference has no counterpart (one process, no
 * collective); NULL is a no-op.
 */
int tq_dp_comm_abort(void* comm);
/*
 * The communicator's asynchronous error (ncclCommGetAsyncError) in
 * *nccl_result: 0 while healthy, an ncclResult_t code once a collective has
 * failed (e.g. a peer's connection closed).  A host that waits for a
 * collective under a deadline polls it beside the collective's completion
 * and aborts the communicator on an error or when the deadline passes.  No
 * reference counterpart (one process, no collective).
 */
int tq_dp_comm_async_error(void* comm, int* nccl_result);

#ifdef __cplusplus
}
#endif

#endif /* TOROBI_B200_H */
