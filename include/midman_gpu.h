/* Kernel-level C ABI of libmidman_gpu.so: the sm_100a kernels behind the
 * training step, callable one at a time on caller-owned device buffers.
 *
 * The reference (MidManStudio/midman-ai) runs these computations as Rust
 * functions over host slices; each entry point below names the reference
 * function it replaces (path:line inside the reference project). A Rust FFI
 * crate (`extern "C"` declarations) or ctypes binds these directly.
 *
 * Conventions
 *   - All pointers are device pointers unless a parameter says "host".
 *   - f32 everywhere; token ids are int32.
 *   - `stream` is a cudaStream_t passed as void* (NULL = the legacy default
 *     stream). Every call is asynchronous on that stream. The GEMM and the
 *     attention forward take their work from two ticket words kept per
 *     (device, stream), so calls on one stream must not be made from two host
 *     threads at once.
 *   - Return value: 0 on success, a negative MM_GPU_ERR_* code otherwise, with a
 *     message from mm_gpu_last_error(). Kernels that wait on hardware pipelines
 *     record timeouts in a device flag read by mm_gpu_device_status().
 *   - Row-major 2-D arrays with an explicit leading dimension in elements.
 */
#ifndef MIDMAN_GPU_H
#define MIDMAN_GPU_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define MM_GPU_EXPORT __attribute__((visibility("default")))
#else
#define MM_GPU_EXPORT
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define MM_GPU_OK 0
#define MM_GPU_ERR_ARGUMENT -1
#define MM_GPU_ERR_SHAPE -3
#define MM_GPU_ERR_INDEX -4
#define MM_GPU_ERR_DEVICE -6

/* Arithmetic of the tensor-core products. */
#define MM_GPU_TF32 0   /* one TF32 pass: ~1e-3 relative error per product */
#define MM_GPU_3XTF32 1 /* hi*hi + hi*lo + lo*hi: close to f32 accuracy */

/* Message of the last failing call on this thread (NUL-terminated, static until
 * the next call). */
MM_GPU_EXPORT const char *mm_gpu_last_error(void);

/* Synchronizes `stream`, returns and clears the device error flag (0 = no
 * kernel reported a timeout). */
MM_GPU_EXPORT int32_t mm_gpu_device_status(void *stream);

/* C[m, n] = sum_k A(m, k) * B(n, k)  (+ R[m, n] when R is not NULL; R may be C).
 * A(m, k) = A[m * lda + k] when a_mn_major == 0 (K-major), A[k * lda + m] when 1.
 * B(n, k) = B[n * ldb + k] when b_mn_major == 0, B[k * ldb + n] when 1.
 * Leading dimensions must be multiples of 4 and pointers 16-byte aligned.
 * Replaces crates/midman-tensor/src/kernels.rs:49-84 (gemm_nn, gemm_nt, gemm_tn)
 * as called from ops_matmul.rs:55-125:
 *   gemm_nn  C = A B     -> a K-major,  b MN-major
 *   gemm_nt  C = A B^T   -> a K-major,  b K-major
 *   gemm_tn  C = A^T B   -> a MN-major, b MN-major */
MM_GPU_EXPORT int32_t mm_gpu_gemm(int32_t m, int32_t n, int32_t k, const float *a, int64_t lda, int32_t a_mn_major,
                    const float *b, int64_t ldb, int32_t b_mn_major, float *c, int64_t ldc,
                    const float *r, int64_t ldr, int32_t precision, void *stream);
/* Global-norm clip and one AdamW step over n_tensors tensors stored one after
 * another in the device arrays p, g, m, v (crates/midman-optim/src/clip.rs:29-59,
 * adamw.rs:141-217): the gradient norm in f64 over a fixed grid (deterministic),
 * gradients scaled by max_norm / (norm + 1e-6) when the norm exceeds max_norm,
 * decoupled decay for the tensors with decay[i] != 0 (the reference decays rank
 * >= 2 tensors), bias corrections in f64 for `step` (1 for the first update).
 * When the norm is not finite nothing changes. norm_out (host, 3 floats):
 * [norm, clip factor, 1 if the update was applied]. Every tensor but the last
 * must hold a multiple of 4 values. Synchronizes the stream. */
MM_GPU_EXPORT int32_t mm_gpu_clip_adamw(int32_t n_tensors, const int64_t *numel, const int32_t *decay, float *p,
                                        const float *g, float *m, float *v, double max_norm, double lr, double beta1,
                                        double beta2, double eps, double weight_decay, uint64_t step,
                                        float *norm_out, void *stream);

/* TF32 sum of products: C = sum over g < nseg of A_g(m, k[g]) B_g(n, k[g])^T (+R),
 * all A_g with one majorness and all B_g with one, summed in one accumulator by a
 * single launch when the shape runs on CTA pairs and nseg <= 3 (otherwise one
 * launch per term accumulating into C). The backward of a layer whose output
 * feeds several projections (dX = dQ Wq^T + dK Wk^T + dV Wv^T) is one call. No
 * counterpart in the reference, which adds the three products through its tape. */
MM_GPU_EXPORT int32_t mm_gpu_gemm_sum(int32_t m, int32_t n, int32_t nseg, const float *const *a, const int64_t *lda,
                                      int32_t a_mn_major, const float *const *b, const int64_t *ldb,
                                      int32_t b_mn_major, const int32_t *k, float *c, int64_t ldc, const float *r,
                                      int64_t ldr, void *stream);

/* Causal grouped-query attention (crates/midman-nn/src/attention.rs:79-102 forward,
 * and its autograd backward). Token-major operands: q, o, dout, dq are
 * [batch * seq, n_heads * head_dim] with row stride ldq (= ldo = lddo = lddq);
 * k, v, dk, dv are [batch * seq, n_kv_heads * head_dim] with row stride ldk.
 * lse and delta are [batch, n_heads, seq]. precision MM_GPU_TF32 runs the score
 * and value products on the tensor cores in the fused flash kernels;
 * MM_GPU_3XTF32 runs them on the tensor cores as three TF32 terms of hi/lo
 * operand pairs through score buffers, the tensor-memory accumulations summed
 * in f32 every 64 values of the contraction (about 4 * batch * n_heads * seq *
 * seq floats of library scratch). The backward forms P from the lse the
 * forward returned. Both need head_dim 32, 64 or 128, row strides multiples of
 * 4 and 16-byte aligned operands; other shapes run the FP32 flash kernels. */
MM_GPU_EXPORT int32_t mm_gpu_attention_forward(int32_t batch, int32_t seq, int32_t n_heads, int32_t n_kv_heads,
                                               int32_t head_dim, const float *q, const float *k, const float *v,
                                               int64_t ldq, int64_t ldk, float *o, float *lse, int32_t precision,
                                               void *stream);
MM_GPU_EXPORT int32_t mm_gpu_attention_backward(int32_t batch, int32_t seq, int32_t n_heads, int32_t n_kv_heads,
                                                int32_t head_dim, const float *q, const float *k, const float *v,
                                                const float *o, const float *lse, const float *dout, int64_t ldq,
                                                int64_t ldk, float *dq, float *dk, float *dv, int32_t precision,
                                                void *stream);

/* ---- The layers around the products (crates/midman-nn, crates/midman-tensor).
 * Token-major activations [rows = batch * seq, features], contiguous unless a
 * row stride is given. Ids and targets outside [0, vocab) are never used to
 * address memory: the host-side checks return MM_GPU_ERR_INDEX, the device-side
 * ones write a zero row (embedding) or a NaN row loss (cross-entropy) and set
 * the device error flag that mm_gpu_device_status reports. */

/* RMSNorm forward (crates/midman-nn/src/norm.rs:21-39): y = x * rstd * w per
 * row, rstd[r] = 1 / sqrt(mean(x[r]^2) + eps) saved for the backward.
 * dim a multiple of 4 up to 8192; x, w, y 16-byte aligned. */
MM_GPU_EXPORT int32_t mm_gpu_rmsnorm_forward(int32_t rows, int32_t dim, const float *x, const float *w, float eps,
                                             float *y, float *rstd, void *stream);
/* RMSNorm backward (the autograd of norm.rs:21-39's six primitives): dx = dres +
 * d(rmsnorm)/dx . dy (dres may be NULL or equal to dx), dw = sum over rows of
 * dy * x * rstd (overwritten), summed in a fixed order (deterministic). */
MM_GPU_EXPORT int32_t mm_gpu_rmsnorm_backward(int32_t rows, int32_t dim, const float *x, const float *w,
                                              const float *rstd, const float *dy, const float *dres, float *dx,
                                              float *dw, void *stream);
/* Rotary embedding in place (crates/midman-nn/src/rope.rs:20-33): x is
 * [rows, heads, head_dim] with row stride ld, rows = batch * seq, row r at
 * position r % seq; each head's halves (x1, x2) become (x1 c - x2 s, x2 c + x1 s)
 * with c, s the rows of the [seq, head_dim / 2] tables (midman_rope_table,
 * rope.rs:54-132). backward != 0 applies the gradient (the rotation by -angle). */
MM_GPU_EXPORT int32_t mm_gpu_rope(int32_t rows, int32_t seq, int32_t heads, int32_t head_dim, float *x, int64_t ld,
                                  const float *cos_t, const float *sin_t, int32_t backward, void *stream);
/* SwiGLU (crates/midman-nn/src/mlp.rs:20-24, silu ops_elementwise.rs:355-364):
 * act = silu(gate) * up over n values. The backward works in place:
 * gate <- dact * up * silu'(gate), up <- dact * silu(gate). */
MM_GPU_EXPORT int32_t mm_gpu_swiglu_forward(int64_t n, const float *gate, const float *up, float *act, void *stream);
MM_GPU_EXPORT int32_t mm_gpu_swiglu_backward(int64_t n, float *gate, float *up, const float *dact, void *stream);
/* Embedding gather (crates/midman-tensor/src/ops_shape.rs:230-255): out[r] =
 * table[ids[r]] with ids on the device; table [vocab, dim], dim a multiple of 4. */
MM_GPU_EXPORT int32_t mm_gpu_embedding_forward(int32_t rows, const int32_t *ids, int32_t vocab, int32_t dim,
                                               const float *table, float *out, void *stream);
/* Embedding scatter-add (ops_shape.rs:262-272): dtable[ids[r]] += dx[r], each
 * table row adding its rows in ascending row order (bit-identical run to run).
 * ids_host is HOST memory: the index that orders the additions is built on the
 * host and copied to the device. Ids outside [0, vocab): MM_GPU_ERR_INDEX,
 * nothing queued. */
MM_GPU_EXPORT int32_t mm_gpu_embedding_backward(int32_t rows, const int32_t *ids_host, int32_t vocab, int32_t dim,
                                                const float *dx, float *dtable, void *stream);
/* Softmax cross-entropy, forward and backward in one pass (crates/midman-tensor/
 * src/ops_reduce.rs:236-276): logits [rows, vocab] (row stride ld) are replaced
 * by grad_scale * (softmax - onehot(target)); row_loss[r] = max + ln(sum exp) -
 * logit[target]; mean_loss (device, may be NULL) receives the mean of row_loss
 * summed in f64 in a fixed order (the reference sums the loss in f64).
 * grad_scale is d(loss)/d(mean), divided by rows (1 / rows for the mean loss). */
MM_GPU_EXPORT int32_t mm_gpu_cross_entropy(int32_t rows, int32_t vocab, float *logits, int64_t ld,
                                           const int32_t *targets, float grad_scale, float *row_loss,
                                           double *mean_loss, void *stream);

/* Failure-path self-test of the bounded waits (no counterpart in the
 * reference): launches one thread that waits on a barrier nothing completes,
 * through the same bounded wait the GEMM and attention pipelines use, limited
 * to timeout_us (1 us .. 10 s). The wait runs out, the kernel records its code
 * in the device error flag and returns, so mm_gpu_device_status reports
 * MM_GPU_ERR_DEVICE ("a bounded wait ran out") and the context stays usable. */
MM_GPU_EXPORT int32_t mm_gpu_wait_selftest(int32_t timeout_us, void *stream);

/* ---- Data-parallel gradient exchange (the step crates/midman-training/src/
 * trainer.rs:162-207 would take between backward and clip with more than one
 * process; the reference is single-process and has no counterpart).
 * One communicator per process and GPU, made from the 128-byte NCCL unique id
 * that rank 0 produced (midman_nccl_unique_id) and shared out of band; create it
 * with the rank's GPU current. */
MM_GPU_EXPORT int32_t mm_gpu_comm_create(const uint8_t *nccl_id, int32_t world, int32_t rank, void **comm_out);
MM_GPU_EXPORT int32_t mm_gpu_comm_destroy(void *comm);
/* In-place all-reduce of one gradient bucket (n floats) across the ranks:
 * the sum, or the mean when average != 0 (equal shards: the gradient of the
 * mean loss over the global batch). Asynchronous on `stream`. */
MM_GPU_EXPORT int32_t mm_gpu_allreduce_bucket(void *comm, float *data, int64_t n, int32_t average, void *stream);
/* Waits for `stream` while polling the communicator for asynchronous NCCL
 * errors. If a peer failed, or the stream has not finished after timeout_ms,
 * the communicator is aborted (its collectives in flight end) and the call
 * returns MM_GPU_ERR_DEVICE; an aborted communicator refuses further use and
 * only mm_gpu_comm_destroy remains. */
MM_GPU_EXPORT int32_t mm_gpu_comm_wait(void *comm, void *stream, int32_t timeout_ms);

/* Allocation-free variant of mm_gpu_attention_forward with precision
 * MM_GPU_TF32 (the tensor-core path; head_dim 32, 64 or 128). No counterpart in
 * the reference, which has no device memory to manage.
 *
 * For callers that cannot let the library call cudaMalloc: a process whose
 * device memory is fully reserved by its own pool (PyTorch's caching
 * allocator, a serving arena) would see the allocation fail, and cudaMalloc /
 * cudaFree can synchronize the device under a caller that overlaps streams.
 * This call allocates nothing: its score scratch is a fixed 16 MiB array inside
 * the library (batch * n_heads * seq * round_up(seq, 4) <= 4194304 floats;
 * larger sizes return MM_GPU_ERR_SHAPE), which every GPU that loads the library
 * holds until the process exits.
 *   - The first call on a device looks up that array's device address (once
 *     per device, with the device current); make it before any stream capture.
 *     The address is kept for the life of the process: do not call this entry
 *     point after a cudaDeviceReset of that device.
 *   - head_dim 32, 64 or 128; ldq and ldk multiples of 4; q, k, v and o 16-byte
 *     aligned (checked before anything is queued).
 *   - All calls share the array: calls whose kernels overlap on the GPU (on
 *     different streams, or from several threads) race on it. Serialize them.
 *   - device_status: device pointer to one int32 that the caller zeroes; the
 *     kernels leave it alone unless a pipeline wait timed out, when it receives
 *     that error code (the codes mm_gpu_device_status reports).
 * Same operands, layouts and results as mm_gpu_attention_forward. */
MM_GPU_EXPORT int32_t mm_gpu_attention_forward_noalloc(int32_t batch, int32_t seq, int32_t n_heads,
                                                       int32_t n_kv_heads, int32_t head_dim, const float *q,
                                                       const float *k, const float *v, int64_t ldq, int64_t ldk,
                                                       float *o, float *lse, int32_t *device_status, void *stream);

#ifdef __cplusplus
}
#endif

#endif
