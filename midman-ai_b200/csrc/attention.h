// Causal grouped-query attention, forward and backward, on token-major
// projections (no head split/merge copies): q [B*T, H, hd] with row stride ldq,
// k and v [B*T, Hkv, hd] with row strides ldk/ldv, o [B*T, H, hd] (ldo).
// Replaces crates/midman-nn/src/attention.rs:79-102 and :146-170 (scores,
// -1e9 mask, softmax, P v, GQA head expansion) and their autograd backward.
#pragma once
#include <cuda_runtime.h>

namespace mm {

struct AttnShape {
  int B, T, H, Hkv, hd;
  long long ldq, ldk, ldv, ldo;
  float scale;  // 1 / sqrt(hd)
};

// o = softmax(q k^T * scale + causal mask) v; lse [B, H, T] = log-sum-exp of each
// scaled score row (natural log), saved for the backward pass.
void attention_forward(const AttnShape& s, const float* q, const float* k, const float* v, float* o, float* lse,
                       cudaStream_t stream);

// Given do (same layout as o), writes dq, dk, dv (dk/dv summed over each key
// head's group of query heads). `delta` is scratch of B*H*T floats.
void attention_backward(const AttnShape& s, const float* q, const float* k, const float* v, const float* o,
                        const float* lse, const float* dout, long long lddo, float* dq, float* dk, float* dv,
                        float* delta, cudaStream_t stream);

// Attention probabilities [B, H, T, T] (zeros above the diagonal), for the
// traced forward (model.rs:116-125, attention.rs:79-85).
void attention_probs(const AttnShape& s, const float* q, const float* k, const float* lse, float* probs,
                     cudaStream_t stream);

// The tensor-core forward through a score buffer (attention_tc.cu), for head_dim
// 32, 64 or 128 in TF32: S holds B*H*T*attention_scores_ld(T) floats. It serves
// the allocation-free entry point, with the pipeline-timeout flag given by the
// caller (no library state).
bool attention_tc_supported(const AttnShape& s);
long long attention_scores_ld(int T);
void attention_forward_tc(const AttnShape& s, const float* q, const float* k, const float* v, float* o, float* lse,
                          float* S, int* d_err, cudaStream_t stream);
// The exact mode on the tensor cores (attention_tc.cu): every product as three
// TF32 terms of hi/lo operand pairs (the operand itself as hi), the
// tensor-memory accumulations restarted every 64 of K and summed in f32, the
// score matrices in `ws` (attention_3x_ws_floats floats: four B*H*T*round4(T)
// matrices, lo copies of q, k, v and dout, and one B*H*T vector). head_dim 32,
// 64 or 128 (attention_tc_supported).
long long attention_3x_ws_floats(const AttnShape& s, long long ld_dout);
void attention_forward_3x(const AttnShape& s, const float* q, const float* k, const float* v, float* o, float* lse,
                          float* ws, int* d_err, cudaStream_t stream);
// The backward takes the forward's lse (P = exp(S * scale - lse)).
void attention_backward_3x(const AttnShape& s, const float* q, const float* k, const float* v, const float* o,
                           const float* lse, const float* dout, long long lddo, float* dq, float* dk, float* dv,
                           float* ws, int* d_err, cudaStream_t stream);
// Fused tensor-core forward (flash_tc.cu): scores stay on chip, no scratch.
// head_dim 32, 64 or 128; row strides multiples of 4; 16-byte aligned pointers.
bool attention_flash_supported(const AttnShape& s);
void attention_forward_flash(const AttnShape& s, const float* q, const float* k, const float* v, float* o,
                             float* lse, int* d_err, cudaStream_t stream);
// A second stream for the backward's dQ kernel, with two events of the caller's:
// the side stream waits for delta, the main stream for the side's kernel.
struct BwdSide {
  cudaStream_t stream;
  cudaEvent_t ready, done;
};
// Fused tensor-core backward (flash_bwd.cu): writes delta (B*H*T floats) and
// dq, dk, dv (dk/dv summed over each key head's group); no score buffers. With
// `side`, the dQ kernel runs beside the dK/dV kernel on side->stream; the work
// is complete on `stream` when the call's work there is.
void attention_backward_flash(const AttnShape& s, const float* q, const float* k, const float* v, const float* o,
                              const float* lse, const float* dout, long long lddo, float* dq, float* dk, float* dv,
                              float* delta, int* d_err, cudaStream_t stream, const BwdSide* side = nullptr);
// delta[b, h, t] = sum_d dout[t, h, d] * o[t, h, d]
void attention_delta(const AttnShape& s, const float* o, const float* dout, long long lddo, float* delta,
                     cudaStream_t stream);

}  // namespace mm
