/*
 * picotron_b200.h -- C ABI of the B200 (sm_100a) RMSNorm / SwiGLU / RoPE hot path and the
 * next-step kernels around it (fused residual add + RMSNorm, SwiGLU fused into the gate/up
 * GEMM, cross-entropy, AdamW).
 *
 * This is the drop-in boundary for picotron's `model.triton_kernels.{rmsnorm,swiglu,rope}`
 * kernels. Every entry point takes plain device pointers, element counts, strides (in
 * elements, not bytes), dtype codes and a CUDA stream passed as `void*` (a cudaStream_t;
 * NULL means the legacy default stream). No entry point allocates device memory except
 * where a comment says so; outputs are written into caller-owned buffers, inputs are
 * read-only. Calls are re-entrant. The state the library shares between calls is:
 *   - per-device caches of device properties and kernel occupancy (written once);
 *   - the thread-local error string returned by pt_last_error();
 *   - per-device error words in device memory, set by a kernel whose bounded wait ran out
 *     and read and cleared by pt_take_device_error();
 *   - the device scratch array of pt_rmsnorm_bwd_noalloc (see there), shared by all its
 *     calls on a device.
 *
 * Work is ordered on the given stream as for any launch. The RMSNorm kernels and the dweight
 * reduce are launched as programmatic dependents of the stream's previous kernel: their CTAs
 * may start while that kernel finishes and wait, before touching global memory, for it to
 * complete, so the ordering seen by the caller is unchanged (also inside CUDA graphs).
 *
 * Every function returns a pt_status. On failure nothing has been launched and
 * pt_last_error() describes the cause on the calling thread. All pointers must be
 * device (or managed) memory of the CUDA device that is current on the calling thread;
 * the library checks this before it launches anything.
 *
 * Reference interfaces replaced (paths inside the picotron project):
 *   src/picotron/nn/triton_kernels/rmsnorm.py  -- triton_rms_norm, _RMSNormAutogradFunction
 *   src/picotron/nn/triton_kernels/swiglu.py   -- triton_swiglu, _SwiGLUAutogradFunction
 *   src/picotron/nn/triton_kernels/rope.py     -- triton_apply_rotary_embedding
 *   src/picotron/nn/rope.py                    -- apply_rotary_embedding (eager fwd + autograd bwd)
 *   src/picotron/utils/hardware.py             -- detect_triton_support (capability probe)
 *   src/picotron/models/picotron_decoder.py    -- residual add + norm of the decoder block
 *   src/picotron/nn/feedforward.py             -- SwiGLU gate/up projections + activation
 *   src/picotron/nn/triton_kernels/cross_entropy.py, training/train_loop.py -- the loss
 *   src/picotron/nn/triton_kernels/adamw.py    -- the (reserved) fused AdamW step
 */
#ifndef PICOTRON_B200_H
#define PICOTRON_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Exported symbols; the library is built with hidden default visibility. */
#if defined(__GNUC__)
#define PT_API __attribute__((visibility("default")))
#else
#define PT_API
#endif

#define PT_ABI_VERSION 1

/* Status codes returned by every entry point. */
enum pt_status {
    PT_OK = 0,
    PT_ERR_INVALID_ARGUMENT = 1, /* null pointer, negative size, bad enum value */
    PT_ERR_UNSUPPORTED_DTYPE = 2, /* dtype code or dtype combination not built */
    PT_ERR_SHAPE = 3,             /* sizes or strides that the op cannot accept */
    PT_ERR_DEVICE = 4,            /* no device, wrong device, pointer not on the current device */
    PT_ERR_CUDA = 5               /* a CUDA runtime call or a kernel launch failed */
};

/* Element types. Values are stable across ABI versions. */
enum pt_dtype {
    PT_FLOAT32 = 0,
    PT_FLOAT16 = 1,
    PT_BFLOAT16 = 2
};

/* RoPE pair layouts. INTERLEAVED rotates (x[2i], x[2i+1]) and is the layout of the
 * reference (src/picotron/nn/rope.py:42-51, triton_kernels/rope.py:40-49).
 * ROTATE_HALF rotates (x[i], x[i + D/2]) (the Llama/HF convention). */
enum pt_rope_layout {
    PT_ROPE_INTERLEAVED = 0,
    PT_ROPE_ROTATE_HALF = 1
};

/* ABI version the library was built with (PT_ABI_VERSION). No reference counterpart. */
PT_API int pt_abi_version(void);

/* Thread-local, NUL-terminated description of the last failure on this thread.
 * Replaces the message of the Triton*Unavailable exceptions
 * (rmsnorm.py:19, swiglu.py:20, triton_kernels/rope.py:19). */
PT_API const char* pt_last_error(void);

/* Capability probe. Fills the compute capability and SM count of `device` and returns
 * PT_OK only when the device can run this library's sm_100a code (compute capability
 * 10.0). Replaces detect_triton_support (src/picotron/utils/hardware.py:93-108), whose
 * check was "triton installed and capability >= 7.0". Any output pointer may be NULL. */
PT_API int pt_probe(int device, int* cc_major, int* cc_minor, int* sm_count);

/* ---------------------------------------------------------------- RMSNorm -------- */

/* y[r, :] = x[r, :] * rsqrt(mean(x[r, :]^2) + eps) * weight, fp32 accumulation, y in the
 * x dtype. rstd (optional, may be NULL) receives rsqrt(mean(x^2) + eps) per row in fp32.
 * Row strides are in elements; the last dimension must be contiguous.
 * Supported (x_dtype, w_dtype): (f32,f32) (f16,f16) (f16,f32) (bf16,bf16) (bf16,f32).
 * Replaces _rmsnorm_kernel + _run_triton_forward + _inverse_rms
 * (src/picotron/nn/triton_kernels/rmsnorm.py:25-84, 49-53). */
PT_API int pt_rmsnorm_fwd(const void* x, int64_t x_row_stride,
                   const void* weight,
                   void* y, int64_t y_row_stride,
                   float* rstd,
                   int64_t rows, int64_t hidden,
                   int x_dtype, int w_dtype, float eps,
                   void* stream);

/* Number of dweight partial rows that pt_rmsnorm_bwd should be given for this problem on
 * the current device: two per resident CTA of the backward kernel (a sum row and an error
 * row). Any positive value is valid; the result of the backward depends only on (inputs,
 * num_partials). */
PT_API int pt_rmsnorm_bwd_num_partials(int64_t rows, int64_t hidden, int x_dtype, int w_dtype,
                                int* num_partials);

/* Backward of pt_rmsnorm_fwd. With r = rsqrt(mean(x^2) + eps) (read from `rstd` when it
 * is not NULL, else recomputed from x) and g = dy * weight:
 *   dx = r * (g - x * r^2 * mean(g * x))              (written in the x dtype)
 *   dw_partials[p, :] + dw_partials[G + p, :] = sum over the rows that CTA p owns of
 *   dy * x * r, as an fp32 (sum, accumulated rounding error) pair, G = num_partials / 2
 *   CTAs (an odd last row is written as zeros; num_partials == 1 gives one CTA whose
 *   rounded total fills row 0).
 * dw_partials is caller-owned scratch of num_partials * hidden floats; every element is
 * written. Reduce it with pt_rmsnorm_dw_reduce. Deterministic for fixed num_partials.
 * dy has the x dtype. Replaces _RMSNormAutogradFunction.backward
 * (src/picotron/nn/triton_kernels/rmsnorm.py:109-134). */
PT_API int pt_rmsnorm_bwd(const void* dy, int64_t dy_row_stride,
                   const void* x, int64_t x_row_stride,
                   const void* weight,
                   const float* rstd,
                   void* dx, int64_t dx_row_stride,
                   float* dw_partials, int num_partials,
                   int64_t rows, int64_t hidden,
                   int x_dtype, int w_dtype, float eps,
                   void* stream);

/* dw[c] = sum over p < num_partials of dw_partials[p, c], fp32, in a summation order that
 * depends only on num_partials (so the result is bit-reproducible), stored in dw_dtype
 * (the weight dtype). Second, deterministic stage of the dweight reduction; replaces
 * `.reshape(-1, H).sum(dim=0)` at rmsnorm.py:125-127. */
PT_API int pt_rmsnorm_dw_reduce(const float* dw_partials, int num_partials, int64_t hidden,
                         void* dw, int dw_dtype, void* stream);

/* Floats of device workspace that pt_rmsnorm_bwd_fused needs for this problem on the
 * current device: a 64-float header, then pt_rmsnorm_bwd_num_partials rows of hidden. */
PT_API int pt_rmsnorm_bwd_fused_workspace(int64_t rows, int64_t hidden, int x_dtype,
                                          int w_dtype, int64_t* floats);

/* pt_rmsnorm_bwd followed by pt_rmsnorm_dw_reduce in one kernel launch: dx (x dtype) and
 * dw (w_dtype) with the same bits as that pair given pt_rmsnorm_bwd_num_partials partial
 * rows. The backward's CTAs, all resident at once (a cooperative launch), write their
 * dweight partial rows into the workspace, meet at a grid barrier and then reduce the
 * partials among themselves in the fixed order of pt_rmsnorm_dw_reduce; this saves the
 * second launch and the partials' trip through a second kernel. Rows the fast pipeline
 * does not take (misaligned, hidden not a multiple of 16 bytes) run the two kernels
 * instead, with the same results.
 * workspace: caller-owned device memory, 256-byte aligned, of at least workspace_floats >=
 * pt_rmsnorm_bwd_fused_workspace floats. Its first word is the grid barrier's counter,
 * whose low 31 bits must be zero before the first call: zero the workspace once after
 * allocating it. Every call that completes leaves the counter that way, so the same
 * workspace serves any number of calls, of any shape, without clearing; after a device
 * error reported by pt_take_device_error, zero it again. Calls that share a workspace must
 * not overlap on the GPU (use one workspace per stream). Replaces
 * _RMSNormAutogradFunction.backward (src/picotron/nn/triton_kernels/rmsnorm.py:109-134). */
PT_API int pt_rmsnorm_bwd_fused(const void* dy, int64_t dy_row_stride,
                                const void* x, int64_t x_row_stride,
                                const void* weight,
                                const float* rstd,
                                void* dx, int64_t dx_row_stride,
                                void* dw,
                                float* workspace, int64_t workspace_floats,
                                int64_t rows, int64_t hidden,
                                int x_dtype, int w_dtype, float eps,
                                void* stream);

/* pt_rmsnorm_bwd without any device allocation, for callers that cannot allocate device
 * memory themselves: a host runtime whose memory pool owns all of the device's memory, a
 * training step that must not pay cudaMalloc/cudaFree's implicit device synchronisation,
 * or a thin FFI binding with no allocator to size and keep a dw_partials buffer. Computes
 * dx (x dtype) and dw (w_dtype) directly. It has no counterpart in the reference.
 * The dweight partials go to a scratch array inside the library (2^22 floats = 16 MiB per
 * device, kept until the process exits); hidden above 2^22 is rejected with PT_ERR_SHAPE.
 * The array holds the partial rows of every CTA pt_rmsnorm_bwd would use on a B200 up to
 * hidden 7085; for wider rows the call runs fewer CTAs than pt_rmsnorm_bwd (as many as
 * the array has rows for) and may be slower, with the same kind of result.
 * The first call on a device looks up that array's address (cudaGetSymbolAddress), so
 * make it before any stream capture; the address is kept for the life of the process, so
 * do not call this entry point after cudaDeviceReset. All calls share the one array: calls whose work
 * overlaps on the GPU (different streams, or different host threads on one device without
 * ordering) race on it and must be serialised by the caller. Nothing in the array needs
 * to start at zero: each call writes every partial it later reads. */
PT_API int pt_rmsnorm_bwd_noalloc(const void* dy, int64_t dy_row_stride,
                                  const void* x, int64_t x_row_stride,
                                  const void* weight,
                                  const float* rstd,
                                  void* dx, int64_t dx_row_stride,
                                  void* dw,
                                  int64_t rows, int64_t hidden,
                                  int x_dtype, int w_dtype, float eps,
                                  void* stream);

/* ------------------------------------------------- fused residual add + RMSNorm -- */

/* h = residual + branch (fp32 add, rounded to the x dtype, written to h_out) and
 * y = h * r * weight with r = rsqrt(mean(h^2) + eps) over the stored (rounded) h, in one
 * pass. Replaces the pair `hidden_states = hidden_states + attention(...)` followed by
 * `self.mlp_norm(hidden_states)` in DecoderBlock.forward_with_auxiliary_loss
 * (src/picotron/models/picotron_decoder.py:116-123), and the block output
 * `hidden_states + mlp_output` followed by the next block's attention_norm: one read of
 * each input and one write of each output instead of an add pass plus a norm pass.
 * residual, branch, h_out and y share x_dtype; h_out may be residual itself (in-place
 * update of the residual stream); y aliases nothing. rstd as in pt_rmsnorm_fwd. */
PT_API int pt_add_rmsnorm_fwd(const void* residual, int64_t residual_row_stride,
                              const void* branch, int64_t branch_row_stride,
                              const void* weight,
                              void* h_out, int64_t h_row_stride,
                              void* y, int64_t y_row_stride,
                              float* rstd,
                              int64_t rows, int64_t hidden,
                              int x_dtype, int w_dtype, float eps,
                              void* stream);

/* Partial rows for pt_add_rmsnorm_bwd (same meaning as pt_rmsnorm_bwd_num_partials). */
PT_API int pt_add_rmsnorm_bwd_num_partials(int64_t rows, int64_t hidden, int x_dtype,
                                           int w_dtype, int* num_partials);

/* Backward of pt_add_rmsnorm_fwd: dx = (RMSNorm backward of dy at h, as pt_rmsnorm_bwd) +
 * dh, rounded once, where dh is the gradient that reaches h through its other use (the
 * residual stream); dx is the gradient of both residual and branch. dw_partials as in
 * pt_rmsnorm_bwd (reduce with pt_rmsnorm_dw_reduce). dx may alias dh; dh == NULL means no
 * other use (plain pt_rmsnorm_bwd). Replaces the autograd of the add + RMSNorm pair at
 * picotron_decoder.py:116-123 (RMSNorm backward, rmsnorm.py:109-134, then the gradient
 * accumulation of the residual add). */
PT_API int pt_add_rmsnorm_bwd(const void* dy, int64_t dy_row_stride,
                              const void* dh, int64_t dh_row_stride,
                              const void* h, int64_t h_row_stride,
                              const void* weight,
                              const float* rstd,
                              void* dx, int64_t dx_row_stride,
                              float* dw_partials, int num_partials,
                              int64_t rows, int64_t hidden,
                              int x_dtype, int w_dtype, float eps,
                              void* stream);

/* Workspace floats of pt_add_rmsnorm_bwd_fused (as pt_rmsnorm_bwd_fused_workspace, with
 * the partial count of pt_add_rmsnorm_bwd_num_partials). */
PT_API int pt_add_rmsnorm_bwd_fused_workspace(int64_t rows, int64_t hidden, int x_dtype,
                                              int w_dtype, int64_t* floats);

/* pt_add_rmsnorm_bwd followed by pt_rmsnorm_dw_reduce in one launch, as
 * pt_rmsnorm_bwd_fused is for pt_rmsnorm_bwd (same workspace contract); dh == NULL is
 * pt_rmsnorm_bwd_fused. */
PT_API int pt_add_rmsnorm_bwd_fused(const void* dy, int64_t dy_row_stride,
                                    const void* dh, int64_t dh_row_stride,
                                    const void* h, int64_t h_row_stride,
                                    const void* weight,
                                    const float* rstd,
                                    void* dx, int64_t dx_row_stride,
                                    void* dw,
                                    float* workspace, int64_t workspace_floats,
                                    int64_t rows, int64_t hidden,
                                    int x_dtype, int w_dtype, float eps,
                                    void* stream);

/* Reads and clears this library's device-side error word of the current device
 * (synchronous: waits for the device). *code = 0 means no kernel reported a problem;
 * 1 means a kernel gave up waiting for one of its own TMA copies or MMAs (after about a
 * second) and skipped the rest of its work, so outputs of the affected call are incomplete;
 * 2 means pt_cross_entropy_fwd met a target outside [0, vocab) that is not ignore_index
 * (its row loss, and so the mean, is NaN).
 * No reference counterpart: the reference has no device-side waits. */
PT_API int pt_take_device_error(int* code);

/* Self-test of the failure path above without a GPU fault: launches one CTA whose thread 0
 * waits on a shared-memory barrier that nothing arrives at, gives up after limit_cycles SM
 * cycles (1 .. 2e9; about 1 ms per 2e6 at 1.9 GHz), records code 1 in the device error word
 * exactly as the pipelines' bounded waits do, and returns, leaving the context usable.
 * No reference counterpart. */
PT_API int pt_selftest_wait_timeout(int64_t limit_cycles, void* stream);

/* ----------------------------------------------------------------- SwiGLU -------- */

/* out = gate * sigmoid(gate) * up over n contiguous elements, fp32 math, one rounding.
 * All three tensors share `dtype`. Replaces _swiglu_kernel + _run_triton_forward
 * (src/picotron/nn/triton_kernels/swiglu.py:26-53). */
PT_API int pt_swiglu_fwd(const void* gate, const void* up, void* out, int64_t n, int dtype,
                  void* stream);

/* s = sigmoid(gate); dgate = dout * up * s * (1 + gate * (1 - s)); dup = dout * gate * s.
 * fp32 math with sigmoid recomputed from gate, one rounding per output. Replaces
 * _SwiGLUAutogradFunction.backward (src/picotron/nn/triton_kernels/swiglu.py:71-81). */
PT_API int pt_swiglu_bwd(const void* dout, const void* gate, const void* up,
                  void* dgate, void* dup, int64_t n, int dtype, void* stream);

/* ------------------------------------------ SwiGLU fused into the gate/up GEMM -- */

/* gate = x @ w_gate^T and up = x @ w_up^T on the tcgen05 tensor cores (fp32 accumulation),
 * each rounded to `dtype`, and act = gate * sigmoid(gate) * up (fp32 math on the rounded
 * values, one rounding) written straight from the accumulators: x [m, k], w_gate and w_up
 * [n, k] (nn.Linear weight layout), act [m, n]; gate_out and up_out [m, n] (row stride
 * pre_row_stride) receive gate and up for the backward, or are both NULL. All matrices are
 * row-major with unit column stride and 16-byte-aligned rows: n, k and every row stride must
 * be multiples of 8. dtype is PT_BFLOAT16 or PT_FLOAT16. Replaces gate_projection,
 * up_projection and the activation of SwiGLU.forward (src/picotron/nn/feedforward.py:27-43;
 * activation at :29-42) up to the down projection. */
PT_API int pt_swiglu_gemm_fwd(const void* x, int64_t x_row_stride,
                              const void* w_gate, const void* w_up, int64_t w_row_stride,
                              void* act, int64_t act_row_stride,
                              void* gate_out, void* up_out, int64_t pre_row_stride,
                              int64_t m, int64_t n, int64_t k, int dtype,
                              void* stream);

/* The training backward of the MLP's activation, fused into the GEMM that produces its input
 * gradient: d_act = dy @ w_down (dy [m, k] the down projection's output gradient, w_down the
 * nn.Linear weight [k, n]) on the tensor cores, and in the epilogue, from gate and up [m, n]
 * as the forward saved them:
 *   dgate = (d_act * up) * (s * (1 + gate * (1 - s))),  dup = d_act * (gate * s),
 *   s = sigmoid(gate), fp32 math on d_act rounded to the dtype, results in the dtype.
 * d_act is stored too when dact_out is not NULL. w_down_t is w_down transposed, [n, k]
 * row-major (both GEMM operands are then read along k). Replaces the autograd of
 * down_projection plus _SwiGLUAutogradFunction.backward (src/picotron/nn/feedforward.py:
 * 27-43, src/picotron/nn/triton_kernels/swiglu.py:71-81): d_act never goes through HBM and
 * the activation backward needs no launch of its own. n (the intermediate size) a multiple of
 * 64, k a multiple of 8, 16-byte aligned pointers and row strides of 8 elements; outputs
 * alias no input. bf16 or fp16. */
PT_API int pt_swiglu_gemm_bwd(const void* dy, int64_t dy_row_stride,
                              const void* w_down_t, int64_t w_row_stride,
                              const void* gate, const void* up, int64_t pre_row_stride,
                              void* dgate, void* dup, int64_t grad_row_stride,
                              void* dact_out, int64_t dact_row_stride,
                              int64_t m, int64_t n, int64_t k, int dtype,
                              void* stream);

/* dst[c, r] = src[r, c] for a [rows, cols] matrix (row strides in elements), in 64 x 64 tiles
 * through shared memory: w_down as [k, n] into the w_down_t that pt_swiglu_gemm_bwd reads.
 * bf16, fp16 or fp32; dst must not alias src. No reference counterpart (the reference's
 * backward multiplies by w_down through autograd without a transposed copy). */
PT_API int pt_transpose_2d(const void* src, int64_t src_row_stride,
                           void* dst, int64_t dst_row_stride,
                           int64_t rows, int64_t cols, int dtype, void* stream);

/* ---------------------------------------------------------- cross-entropy ------- */

/* Mean cross-entropy over rows of `vocab` logits (class stride 1). Rows form an
 * [outer, inner] grid: row (o, i) starts at logits + o * logits_outer_stride +
 * i * logits_inner_stride and its target is targets[o * targets_outer_stride +
 * i * targets_inner_stride] (int64); strides are in elements. So the training call
 * F.cross_entropy(logits[:, :-1, :].transpose(1, 2), input_ids[:, 1:]) reads [B, S, V] logits
 * in place with outer = B, inner = S - 1, strides (S * V, V) and targets (S, 1) from
 * input_ids + 1. Writes row_loss[r] = lse_r - x_r[target] (0 for ignore_index rows) and
 * row_lse[r] = log(sum(exp(x_r))) (fp32, dense [rows]), then mean_out[0] = the mean of
 * row_loss over the rows whose target is not ignore_index and mean_out[1] = 1 / their count
 * (NaN for both when there are none), deterministically. fp32 math from f32/f16/bf16 logits.
 * Replaces the loss of src/picotron/training/train_loop.py:95-97,141-145 (F.cross_entropy,
 * mean reduction) and the forward-only Triton kernel of
 * src/picotron/nn/triton_kernels/cross_entropy.py:28-87. */
PT_API int pt_cross_entropy_fwd(const void* logits, int64_t vocab, int64_t outer,
                                int64_t inner, int64_t logits_outer_stride,
                                int64_t logits_inner_stride, const int64_t* targets,
                                int64_t targets_outer_stride, int64_t targets_inner_stride,
                                int64_t ignore_index, float* row_loss, float* row_lse,
                                float* mean_out, int dtype, void* stream);

/* Gradient of pt_cross_entropy_fwd's mean loss: dlogits = (softmax(x_r) - onehot(target_r))
 * * grad_loss * mean_out[1] (grad_loss: one fp32 value in device memory, or NULL for 1),
 * zeros for ignored rows, written in the logits dtype at dlogits with its own two row
 * strides (class stride 1). Recomputes softmax from row_lse. Replaces the autograd
 * backward of F.cross_entropy at train_loop.py:141-145. */
PT_API int pt_cross_entropy_bwd(const void* logits, int64_t vocab, int64_t outer,
                                int64_t inner, int64_t logits_outer_stride,
                                int64_t logits_inner_stride, const int64_t* targets,
                                int64_t targets_outer_stride, int64_t targets_inner_stride,
                                int64_t ignore_index, const float* row_lse,
                                const float* mean_out, const float* grad_loss, void* dlogits,
                                int64_t dlogits_outer_stride, int64_t dlogits_inner_stride,
                                int dtype, void* stream);

/* ------------------------------------------------------------------ AdamW -------- */

/* One fused AdamW step over num_tensors fp32 parameters (device pointers in host arrays):
 * for tensor i, numels[i] elements of params[i], grads[i], exp_avgs[i] and exp_avg_sqs[i]
 * (same layout, dense), at step steps[i] (the count after this step's increment, >= 1), with
 * learning rate lrs[i] and weight decay weight_decays[i] (its parameter group's values).
 * Computes torch.optim.AdamW's update (decoupled weight decay, amsgrad off, maximize as
 * given) with the same fp32 operations and roundings as its CUDA multi-tensor path, so the
 * results are bit-identical to it, in one read and one write of each array. Replaces the
 * reserved fused-AdamW extension point of src/picotron/nn/triton_kernels/adamw.py:14-24
 * (called from src/picotron/training/train_loop.py:98-100,168), whose fallback is that
 * torch.optim.AdamW (train_loop.py:302-325). */
PT_API int pt_adamw_step(float* const* params, const float* const* grads,
                         float* const* exp_avgs, float* const* exp_avg_sqs,
                         const int64_t* numels, const int64_t* steps, const double* lrs,
                         const double* weight_decays, int num_tensors, double beta1,
                         double beta2, double eps, int maximize, void* stream);

/* ------------------------------------------------------------------- RoPE -------- */

/* Rotary embedding of a 4-D tensor with logical shape sizes = [B, H, S, D] (the
 * reference's (batch, heads, sequence, head_dim) view) and arbitrary strides in elements
 * for x and out (stride of D must be 1). The angle of pair i at sequence index s comes
 * from the tables cosine/sine of logical shape [S, D/2] with row stride table_row_stride
 * (elements) and contiguous columns, in table_dtype. INTERLEAVED:
 *   out[2i]   = x[2i] * c - x[2i+1] * s,   out[2i+1] = x[2i] * s + x[2i+1] * c
 * fp32 math, one rounding. Replaces apply_rotary_embedding (src/picotron/nn/rope.py:35-51)
 * and triton_apply_rotary_embedding (src/picotron/nn/triton_kernels/rope.py:52-91). */
PT_API int pt_rope_fwd(const void* x, const int64_t x_strides[4],
                void* out, const int64_t out_strides[4],
                const int64_t sizes[4],
                const void* cosine, const void* sine, int64_t table_row_stride,
                int layout, int dtype, int table_dtype, void* stream);

/* Backward of pt_rope_fwd: the rotation by -angle (the transpose of the forward
 * rotation), i.e. for INTERLEAVED
 *   dx[2i] = dy[2i] * c + dy[2i+1] * s,   dx[2i+1] = -dy[2i] * s + dy[2i+1] * c.
 * Replaces the autograd backward of apply_rotary_embedding (src/picotron/nn/rope.py:35-51),
 * which the reference's Triton kernel does not provide (triton_kernels/rope.py:60-61). */
PT_API int pt_rope_bwd(const void* dy, const int64_t dy_strides[4],
                void* dx, const int64_t dx_strides[4],
                const int64_t sizes[4],
                const void* cosine, const void* sine, int64_t table_row_stride,
                int layout, int dtype, int table_dtype, void* stream);

/* pt_rope_fwd / pt_rope_bwd of a query and a key tensor that share head_dim, the sequence
 * length and the tables, in one launch (the pair RotaryEmbedding.forward rotates,
 * src/picotron/nn/rope.py:70-107). Each tensor has its own sizes and strides, as above. */
PT_API int pt_rope_qk_fwd(const void* q, const int64_t q_strides[4], void* q_out,
                          const int64_t q_out_strides[4], const int64_t q_sizes[4],
                          const void* k, const int64_t k_strides[4], void* k_out,
                          const int64_t k_out_strides[4], const int64_t k_sizes[4],
                          const void* cosine, const void* sine, int64_t table_row_stride,
                          int layout, int dtype, int table_dtype, void* stream);
PT_API int pt_rope_qk_bwd(const void* dq, const int64_t dq_strides[4], void* dq_out,
                          const int64_t dq_out_strides[4], const int64_t q_sizes[4],
                          const void* dk, const int64_t dk_strides[4], void* dk_out,
                          const int64_t dk_out_strides[4], const int64_t k_sizes[4],
                          const void* cosine, const void* sine, int64_t table_row_stride,
                          int layout, int dtype, int table_dtype, void* stream);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* PICOTRON_B200_H */
