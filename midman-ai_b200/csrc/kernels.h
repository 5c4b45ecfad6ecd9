// Launchers of the bandwidth-bound kernels of the training step (kernels.cu,
// attention.cu, optim.cu). All are asynchronous on `stream`; sizes in elements.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

namespace mm {

// ---- embedding (crates/midman-tensor/src/ops_shape.rs:230-275)
// out[r] = table[ids[r]]; an id outside [0, vocab) gives a zero row and sets *err
// (when err is not null) to kErrIndex.
void embedding_forward(const int32_t* ids, int rows, const float* table, int vocab, int dim, float* out, int* err,
                       cudaStream_t s);
// Deterministic scatter-add in the reference's order: for every distinct id u,
// dtable[ids_u] += dx[p] for its positions p in ascending order (CSR on the host).
void embedding_backward(const int32_t* uniq, const int32_t* offsets, const int32_t* positions, int n_uniq,
                        const float* dx, int dim, float* dtable, cudaStream_t s);

// ---- RMSNorm (crates/midman-nn/src/norm.rs:21-39)
// y = x * rstd * w with rstd = 1 / sqrt(mean(x^2) + eps), saved per row.
void rmsnorm_forward(const float* x, const float* w, int rows, int dim, float eps, float* y, float* rstd,
                     cudaStream_t s);
// dx = dres + dNorm/dx . dy (dres may be null or alias dx); dw = sum over rows (overwritten).
// `ws` must hold rmsnorm_ws_floats(rows, dim) floats.
void rmsnorm_backward(const float* x, const float* w, const float* rstd, const float* dy, int rows, int dim,
                      float* dx, const float* dres, float* dw, float* ws, cudaStream_t s);
long long rmsnorm_ws_floats(int rows, int dim);

// ---- rotary embedding (crates/midman-nn/src/rope.rs:20-33, 114-132)
// x: token-major [rows = B*T, heads, hd] with row stride `ld`; position = row % T.
// forward rotates by +angle, backward (the gradient) by -angle.
void rope(float* x, int rows, int T, int heads, int hd, long long ld, const float* cos_t, const float* sin_t,
          bool backward, cudaStream_t s);

// ---- SwiGLU (crates/midman-nn/src/mlp.rs:20-24)
void swiglu_forward(const float* g, const float* u, float* act, long long n, cudaStream_t s);
// In place: g <- d/dg, u <- d/du given dact.
void swiglu_backward(float* g, float* u, const float* dact, long long n, cudaStream_t s);

// ---- softmax cross-entropy (crates/midman-tensor/src/ops_reduce.rs:236-276)
// In place: logits <- d(mean loss)/d logits (scale = 1/total_rows); row_loss[r] = max + ln(sum) - z_t.
// A target outside [0, vocab) gives a NaN row loss and sets *err (when not null) to kErrIndex.
void cross_entropy(float* logits, long long ld, const int32_t* targets, int rows, int vocab, float grad_scale,
                   float* row_loss, int* err, cudaStream_t s);
// loss_out[0] = sum(row_loss) / rows accumulated in f64 in a fixed order.
void mean_loss(const float* row_loss, int rows, double* loss_out, cudaStream_t s);
// Top-1 prediction per row (first index of the maximum, as lab.rs:300-302).
void argmax_rows(const float* logits, long long ld, int rows, int vocab, int32_t* out, cudaStream_t s);

// ---- global norm, clip and AdamW (crates/midman-optim/src/{clip,adamw}.rs)
struct AdamChunk {
  long long offset;
  int length;
  int decay;  // parameter has rank >= 2
};
// Partial sums of g^2 in f64 (fixed grid: deterministic). partials: kNormBlocks doubles.
// Block b reduces elements [b * norm_block_elems(n), (b + 1) * norm_block_elems(n)) ∩ [0, n);
// with [lo, hi) given, blocks whose range is not inside it write 0 (a data-parallel
// rank's share of the grid: summed over ranks, the partials are the whole grid's).
constexpr int kNormBlocks = 1184;  // 8 x 148 SMs
__host__ __device__ inline long long norm_block_elems(long long n) {
  return ((n + kNormBlocks - 1) / kNormBlocks + 3) & ~3ll;
}
void sumsq_partials(const float* g, long long n, double* partials, cudaStream_t s, long long lo = 0,
                    long long hi = -1);
// status[0..]: finishes the norm from the partials, applies the reference's clip
// rule and writes [norm (f32), clip factor, ok flag] into `norm_out` (device).
void finish_norm(const double* partials, const double* loss, float max_norm, float* norm_out, cudaStream_t s);
// One AdamW step over every chunk, skipped entirely when norm_out says the loss or
// the norm was not finite. Gradients are scaled by the clip factor first. m and v
// hold the moments of the flat elements from mv_base on (chunks lie inside them).
void adamw_step(const AdamChunk* chunks, int n_chunks, float* p, const float* g, float* m, float* v,
                long long mv_base, const float* norm_out, float lr, float beta1, float beta2, float eps,
                float weight_decay, float step_size, float bias2_sqrt, cudaStream_t s);
// Per-tensor sum of squares in f64 (for per-parameter statistics).
void tensor_sumsq(const float* x, long long n, double* out, cudaStream_t s);

// ---- misc
void add(const float* a, const float* b, float* out, long long n, cudaStream_t s);
void scale(float* x, float factor, long long n, cudaStream_t s);

}  // namespace mm
