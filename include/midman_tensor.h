/* Device tensors with a recording autograd tape: the midman-tensor Tensor /
 * Tensor::backward API with the values in GPU memory (libmidman_gpu.so).
 *
 * crates/midman-tensor keeps values in host memory and records a graph node for
 * every operation with an input that tracks gradients (autograd.rs:27-41);
 * Tensor::backward orders the nodes, seeds the output with 1 and runs each
 * node's backward toward the leaves, summing gradients that reach a tensor
 * through several uses (autograd.rs:44-124). Here a tape owns a CUDA stream and
 * the tensors made on it: every operation runs its kernels at once on that
 * stream and, when an input tracks gradients, records its backward;
 * mm_tape_backward replays the records in reverse and leaves each leaf's
 * gradient on the device until read with mm_tensor_grad.
 *
 * Operations are this library's fused layer kernels (tcgen05 GEMMs, RMSNorm,
 * RoPE, SwiGLU, causal flash attention, cross-entropy), so a model's graph has
 * a node per layer operation. Shapes are row-major; widths that a GEMM or a
 * 128-bit kernel reads (matmul inner/output widths, embedding and norm widths)
 * must be multiples of 4.
 *
 * Handles: a tape is a uint32 (0 = failure), a tensor a uint64 within its tape
 * (0 = failure); the message of a failure is mm_gpu_last_error(). Status
 * returns use the MM_GPU_* codes of midman_gpu.h. A tape belongs to the device
 * that was current when it was made; call it with that device current. Tapes
 * are not for concurrent use from several host threads.
 */
#ifndef MIDMAN_TENSOR_H
#define MIDMAN_TENSOR_H

#include <stdint.h>

#include "midman_gpu.h"

#ifdef __cplusplus
extern "C" {
#endif

/* A tape on the current device; its products run in MM_GPU_TF32 or
 * MM_GPU_3XTF32 (the latter with the FP32 attention kernels). */
MM_GPU_EXPORT uint32_t mm_tape_create(int32_t precision);
/* Frees the tape, its tensors and their gradients. */
MM_GPU_EXPORT int32_t mm_tape_destroy(uint32_t tape);

/* Tensor::from_vec / Parameter: a tensor of `rank` (1..4) dimensions, filled from
 * host_values (HOST memory, shape's product of floats) or with zeros when NULL.
 * requires_grad != 0 makes it a leaf whose gradient backward keeps. */
MM_GPU_EXPORT uint64_t mm_tensor_new(uint32_t tape, const int64_t *shape, int32_t rank, const float *host_values,
                                     int32_t requires_grad);
MM_GPU_EXPORT int32_t mm_tensor_shape(uint32_t tape, uint64_t tensor, int64_t *shape_out /* 4 */, int32_t *rank_out);
/* Tensor::data: copies the n values to HOST memory (n must equal the size). */
MM_GPU_EXPORT int32_t mm_tensor_read(uint32_t tape, uint64_t tensor, float *host_out, int64_t n);
/* Grads::get after mm_tape_backward: the leaf's gradient, zeros if none reached it. */
MM_GPU_EXPORT int32_t mm_tensor_grad(uint32_t tape, uint64_t tensor, float *host_out, int64_t n);
/* Drops the caller's handle; nodes recorded on it keep its values while needed. */
MM_GPU_EXPORT int32_t mm_tensor_free(uint32_t tape, uint64_t tensor);
/* Tensor::backward (autograd.rs:69-124) from a single-value tensor that tracks
 * gradients; replaces the gradients of the previous backward. Synchronizes. */
MM_GPU_EXPORT int32_t mm_tape_backward(uint32_t tape, uint64_t loss);

/* a [m, k] x b [k, n] (or b [n, k] read transposed when b_transposed != 0, the
 * tied head's x E^T): ops_matmul.rs:55-75, kernels.rs:49-84. */
MM_GPU_EXPORT uint64_t mm_op_matmul(uint32_t tape, uint64_t a, uint64_t b, int32_t b_transposed);
/* Same-shape sum and product (ops_elementwise.rs:249, :287). */
MM_GPU_EXPORT uint64_t mm_op_add(uint32_t tape, uint64_t a, uint64_t b);
MM_GPU_EXPORT uint64_t mm_op_mul(uint32_t tape, uint64_t a, uint64_t b);
/* Rows of table [vocab, dim] picked by ids (HOST, `rows` of them): ops_shape.rs:230-275. */
MM_GPU_EXPORT uint64_t mm_op_embedding(uint32_t tape, uint64_t table, const int32_t *ids_host, int64_t rows);
/* RMSNorm over the last dimension of x [rows, dim] with weight w [dim]: norm.rs:21-39. */
MM_GPU_EXPORT uint64_t mm_op_rms_norm(uint32_t tape, uint64_t x, uint64_t w, float eps);
/* Rotate-half RoPE of x [batch * seq, heads * head_dim], row r at position r % seq,
 * tables of RotaryTables::new(head_dim, seq, theta): rope.rs:20-132. */
MM_GPU_EXPORT uint64_t mm_op_rope(uint32_t tape, uint64_t x, int32_t seq, int32_t heads, float theta);
/* Causal grouped-query attention of token-major q [batch * seq, n_heads * hd] and
 * k, v [batch * seq, n_kv_heads * hd], scale 1/sqrt(hd): attention.rs:79-170. */
MM_GPU_EXPORT uint64_t mm_op_causal_attention(uint32_t tape, uint64_t q, uint64_t k, uint64_t v, int32_t batch,
                                              int32_t seq, int32_t n_heads, int32_t n_kv_heads);
/* silu(gate) * up (mlp.rs:20-24). */
MM_GPU_EXPORT uint64_t mm_op_swiglu(uint32_t tape, uint64_t gate, uint64_t up);
/* Mean cross-entropy of logits [rows, classes] against targets (HOST), a [1]
 * tensor; the loss is summed in f64 (ops_reduce.rs:236-276). */
MM_GPU_EXPORT uint64_t mm_op_cross_entropy(uint32_t tape, uint64_t logits, const int32_t *targets_host, int64_t rows);

#ifdef __cplusplus
}
#endif

#endif
