/* CPU oracle for the MidMan training step -- TEST INFRASTRUCTURE ONLY.
 *
 * A C++ restatement of the reference's CPU f32 algorithm (MidManStudio/midman-ai,
 * pure Rust, single-threaded), written from its source so that the GPU path can be
 * checked against it. Only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline leg may load it, and only as the checker or the timed CPU baseline;
 * the product (libmidman_gpu.so) never links or calls it.
 *
 * Each function cites the reference file:line it follows. Arithmetic follows the
 * reference's op order: f32 with separate multiply and add (built with
 * -ffp-contract=off), glibc expf/logf/powf as Rust's f32 methods use on Linux,
 * and f64 exactly where the reference accumulates in f64. Output elements may be
 * computed on several threads (OpenMP) without changing any element's own order
 * of operations. The pins against the reference's own known answers live in
 * tests/test_oracle_pins.py.
 */
#ifndef MIDMAN_ORACLE_H
#define MIDMAN_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- Rng: crates/midman-foundation/src/rng.rs:16-119 ---- */
void *or_rng_new(uint64_t seed);
void or_rng_free(void *rng);
uint64_t or_rng_next_u64(void *rng);
float or_rng_next_f32(void *rng);
double or_rng_next_f64(void *rng);
float or_rng_uniform(void *rng, float lo, float hi);
float or_rng_normal(void *rng);
uint64_t or_rng_below(void *rng, uint64_t n);
void or_rng_shuffle(void *rng, uint64_t *items, size_t n);
void *or_rng_fork(void *rng, uint64_t stream);

/* ---- ModelConfig: crates/midman-model-config/src/config.rs:106-183 ----
 * cfg = [vocab, d_model, n_layers, n_heads, n_kv_heads, d_ff, max_seq_len, rope_theta,
 *        norm_eps, tie_embeddings]. out = [embedding, attention, mlp, norms, lm_head, total].
 * Returns 0, or -2 with the offending field's name in msg. */
int or_param_breakdown(const double *cfg, uint64_t *out, char *msg, size_t msg_cap);

/* RotaryTables::new, crates/midman-nn/src/rope.rs:54-85. */
int or_rope_table(int head_dim, int max_seq_len, float theta, float *cos_out, float *sin_out);

/* ---- MidManModel: crates/midman-model/src/model.rs ---- */
/* Builds the model drawing from `rng` in the reference order (model.rs:51-84). */
void *or_model_new(const double *cfg, void *rng, float init_std);
void or_model_free(void *model);
size_t or_model_num_params(void *model);
int or_model_num_tensors(void *model);
/* Name, rank, shape (up to 2 dims), offset and length of parameter `i` in the flat order of
 * MidManModel::parameters (model.rs:187-197). */
int or_model_param_info(void *model, int i, char *name, size_t name_cap, int *rank, int64_t *shape,
                        uint64_t *offset, uint64_t *numel);
void or_model_get_params(void *model, float *out);
void or_model_set_params(void *model, const float *in);

/* Mean next-token cross-entropy (model.rs:174-183). With grads != NULL also runs the backward
 * pass and writes d loss / d param in flat parameter order. Returns 0 or a negative code. */
int or_model_loss(void *model, const int32_t *inputs, const int32_t *targets, int batch, int seq,
                  float *loss, float *grads);
/* Logits [batch * seq, vocab] (model.rs:127-165). */
int or_model_logits(void *model, const int32_t *inputs, int batch, int seq, float *logits);
/* Attention probabilities of every layer, [layers, batch, heads, seq, seq] (model.rs:116-125). */
int or_model_attention(void *model, const int32_t *inputs, int batch, int seq, float *probs);

/* ---- Optimizer: crates/midman-optim ---- */
/* global_norm + clip_global_norm (clip.rs:29-59). Returns the norm before clipping; *ok = 0 when
 * the norm is not finite (nothing modified). */
float or_clip_global_norm(float *grads, size_t n, float max_norm, int *ok);
/* WarmupCosine::lr (schedule.rs:54-64). */
float or_schedule_lr(float max_lr, float min_lr, uint64_t warmup, uint64_t total, uint64_t step);
/* AdamW (adamw.rs:141-217) over the model's parameters, moments in parameter order. */
void *or_adamw_new(void *model, float beta1, float beta2, float eps, float weight_decay);
void or_adamw_free(void *opt);
int or_adamw_step(void *opt, void *model, const float *grads, float lr);
uint64_t or_adamw_steps(void *opt);
void or_adamw_moments(void *opt, float *m, float *v);

/* One Trainer::update (crates/midman-training/src/trainer.rs:185-207): loss, backward, clip,
 * AdamW with the given lr. out = [loss, grad_norm]. Returns 0, or -1 when the loss or the
 * gradient norm is not finite (nothing changed). */
int or_train_update(void *model, void *opt, const int32_t *inputs, const int32_t *targets,
                    int batch, int seq, float clip_norm, float lr, float *out);

/* ---- Data: crates/midman-data/src/batch.rs ---- */
/* Sequences over one shard of `n` tokens cut into windows of seq+1 every seq tokens, and a
 * Batcher of `batch` rows seeded by `seed` (batch.rs:45-248). */
void *or_batcher_new(const uint32_t *tokens, size_t n, int seq, int batch, uint64_t seed);
void or_batcher_free(void *b);
size_t or_batcher_num_sequences(void *b);
/* inputs/targets: batch * seq ids each. Writes epoch and index of the batch. */
void or_batcher_next(void *b, int32_t *inputs, int32_t *targets, uint64_t *epoch, uint64_t *index);

/* ---- Single-op known-answer entry points ---- */
/* kernels.rs:87-109 and :66-75. gemm_tn: C[m,n] += A[k,m]^T B[k,n]. */
void or_gemm_nn(const float *a, const float *b, float *c, size_t m, size_t k, size_t n);
void or_gemm_nt(const float *a, const float *b, float *c, size_t m, size_t k, size_t n);
void or_gemm_tn(const float *a, const float *b, float *c, size_t k, size_t m, size_t n);
/* ops_reduce.rs:97-126 (contiguous path). */
void or_softmax_rows(const float *x, float *y, size_t rows, size_t cols);
/* ops_reduce.rs:236-276: mean loss; grad (nullable) = d loss / d logits. */
float or_cross_entropy(const float *logits, const int32_t *targets, size_t n, size_t v, float *grad);
/* causal_attention (attention.rs:98-102): q [B,H,T,hd], k/v [B,Hkv,T,hd] -> out [B,H,T,hd],
 * probs [B,H,T,T] (nullable). Head counts and head_dim from cfg. */
int or_causal_attention(const double *cfg, const float *q, const float *k, const float *v, int batch, int seq,
                        float *out, float *probs);
/* One AdamW update of one parameter (adamw.rs:192-215). */
int or_adamw_update(float *x, const float *g, float *m, float *v, size_t n, int decay, uint64_t step, float lr,
                    float beta1, float beta2, float eps, float weight_decay);

/* Threads the oracle uses for its parallel loops (0 = OpenMP default). */
void or_set_threads(int n);

#ifdef __cplusplus
}
#endif

#endif
