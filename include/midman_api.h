/* The midman C ABI, served by libmidman_gpu.so: the reference's lab API (same
 * functions, same arguments, same status codes and buffer rules, version 1) plus
 * training entry points for models beyond the lab's limits.
 *
 * Each function replaces the export of the same name in the reference's
 * crates/midman-api/src/ffi.rs (line numbers below); its header is
 * crates/midman-api/ffi-smoke-test/midman_api.h. The only difference a caller
 * sees is where the work runs: every lab and training step executes on the GPU
 * (sm_100a), and results come back into the same library-owned buffers.
 *
 * Boundary rules (unchanged from the reference, ffi.rs:7-25):
 *   - Handles, not pointers: labs and trainers live in the library; a stale or
 *     invented handle is MIDMAN_ERR_ARGUMENT, never undefined behaviour.
 *   - Callers own inputs (8-byte aligned; midman_alloc/midman_free with the same
 *     length), the library owns results: midman_text_*, midman_floats_*,
 *     midman_error_* stay valid until the next call that is not an accessor.
 *   - Status codes only; no C++ exception crosses the boundary (MIDMAN_ERR_PANIC
 *     is returned for anything unexpected, as for a caught panic).
 *   - One thread: state is thread-local, a handle is valid only on its thread.
 *
 * Arrays of numbers are doubles: a model config is MIDMAN_CONFIG_LEN values, a
 * hyperparameter set MIDMAN_HYPER_LEN values, in the enum orders below.
 */
#ifndef MIDMAN_API_H
#define MIDMAN_API_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define MIDMAN_EXPORT __attribute__((visibility("default")))
#else
#define MIDMAN_EXPORT
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define MIDMAN_ABI_VERSION 1u

#define MIDMAN_OK 0
#define MIDMAN_STOPPED 1
#define MIDMAN_ERR_ARGUMENT -1
#define MIDMAN_ERR_CONFIG -2
#define MIDMAN_ERR_SHAPE -3
#define MIDMAN_ERR_INDEX -4
#define MIDMAN_ERR_OTHER -5
/* New code (additions do not change the ABI version): a CUDA or NCCL failure. */
#define MIDMAN_ERR_DEVICE -6
#define MIDMAN_ERR_PANIC -99

#define MIDMAN_CONFIG_LEN 10
#define MIDMAN_HYPER_LEN 8

enum midman_config_field {
  MIDMAN_CONFIG_VOCAB_SIZE = 0,
  MIDMAN_CONFIG_D_MODEL,
  MIDMAN_CONFIG_N_LAYERS,
  MIDMAN_CONFIG_N_HEADS,
  MIDMAN_CONFIG_N_KV_HEADS,
  MIDMAN_CONFIG_D_FF,
  MIDMAN_CONFIG_MAX_SEQ_LEN,
  MIDMAN_CONFIG_ROPE_THETA,
  MIDMAN_CONFIG_NORM_EPS,
  MIDMAN_CONFIG_TIE_EMBEDDINGS
};

enum midman_hyper_field {
  MIDMAN_HYPER_MAX_LR = 0,
  MIDMAN_HYPER_MIN_LR,
  MIDMAN_HYPER_WARMUP_STEPS,
  MIDMAN_HYPER_TOTAL_STEPS,
  MIDMAN_HYPER_WEIGHT_DECAY,
  MIDMAN_HYPER_CLIP_NORM,
  MIDMAN_HYPER_BETA1,
  MIDMAN_HYPER_BETA2
};

/* ---- memory and results (ffi.rs:253-339) ---- */
MIDMAN_EXPORT uint32_t midman_abi_version(void);                 /* ffi.rs:253 */
MIDMAN_EXPORT uint8_t *midman_alloc(uint32_t len);               /* ffi.rs:262 */
MIDMAN_EXPORT void midman_free(uint8_t *ptr, uint32_t len);      /* ffi.rs:278 */
MIDMAN_EXPORT const uint8_t *midman_text_ptr(void);              /* ffi.rs:293 */
MIDMAN_EXPORT uint32_t midman_text_len(void);                    /* ffi.rs:299 */
MIDMAN_EXPORT const float *midman_floats_ptr(void);              /* ffi.rs:306 */
MIDMAN_EXPORT uint32_t midman_floats_len(void);                  /* ffi.rs:312 */
MIDMAN_EXPORT const uint8_t *midman_error_ptr(void);             /* ffi.rs:318 */
MIDMAN_EXPORT uint32_t midman_error_len(void);                   /* ffi.rs:324 */

/* ---- stateless calls (ffi.rs:333-443) ---- */
MIDMAN_EXPORT int32_t midman_describe(void);                               /* ffi.rs:333 */
MIDMAN_EXPORT int32_t midman_preset_config(uint32_t index, double *out);   /* ffi.rs:378 */
MIDMAN_EXPORT int32_t midman_config_report(const double *config);          /* ffi.rs:403 */
MIDMAN_EXPORT int32_t midman_rope_table(uint32_t head_dim, uint32_t max_seq_len, double theta); /* ffi.rs:442 */

/* ---- labs (ffi.rs:473-647): a model, AdamW and a fixed random task ---- */
MIDMAN_EXPORT uint32_t midman_lab_create(const double *config, const double *hyper, uint32_t seed_lo,
                                         uint32_t seed_hi, uint32_t batch, uint32_t seq); /* ffi.rs:473 */
MIDMAN_EXPORT int32_t midman_lab_step(uint32_t handle, uint32_t steps);         /* ffi.rs:518 */
MIDMAN_EXPORT int32_t midman_lab_eval(uint32_t handle);                         /* ffi.rs:539 */
MIDMAN_EXPORT int32_t midman_lab_stats(uint32_t handle);                        /* ffi.rs:576 */
MIDMAN_EXPORT int32_t midman_lab_attention(uint32_t handle, uint32_t sequence); /* ffi.rs:608 */
MIDMAN_EXPORT int32_t midman_lab_embedding(uint32_t handle);                    /* ffi.rs:626 */
MIDMAN_EXPORT int32_t midman_lab_destroy(uint32_t handle);                      /* ffi.rs:641 */

/* ---- training (additions; no counterpart in the reference's ABI, which caps
 * models at 8,000,000 parameters and tasks at 4,096 tokens, lab.rs:22-25).
 * They expose Trainer::step (crates/midman-training/src/trainer.rs:162-207) for
 * any model size, data-parallel over `world` processes (one GPU each). ---- */

/* Arithmetic of the tensor-core products. */
#define MIDMAN_PRECISION_TF32 0
#define MIDMAN_PRECISION_3XTF32 1

/* Writes a new NCCL unique id (128 bytes) for rank 0 to share with the others. */
MIDMAN_EXPORT int32_t midman_nccl_unique_id(uint8_t *out128);

/* Creates a trainer on the current CUDA device. Weights are drawn from the
 * seeded generator exactly as MidManModel::new draws them (model.rs:51-84), init
 * std 0.02. `hyper` as for labs except MIDMAN_HYPER_* warmup/total drive
 * WarmupCosine; AdamW eps is 1e-8. batch x seq is this rank's share of a step.
 * world > 1 needs `nccl_id` (128 bytes, identical on every rank). Returns a
 * handle, or 0 with the reason in the error buffer. */
MIDMAN_EXPORT uint32_t midman_train_create(const double *config, const double *hyper, uint32_t seed_lo,
                                           uint32_t seed_hi, uint32_t batch, uint32_t seq, uint32_t precision,
                                           uint32_t world, uint32_t rank, const uint8_t *nccl_id);
/* One step on this rank's ids (batch*seq int32 inputs and targets). Numeric
 * result: [loss, grad_norm, lr]. MIDMAN_STOPPED if the loss or the gradient
 * norm was not finite (nothing changed). */
MIDMAN_EXPORT int32_t midman_train_step(uint32_t handle, const int32_t *inputs, const int32_t *targets);
/* Copies a batch to the device once; midman_train_step_staged then runs
 * `steps` steps on it (inputs resident in HBM). Numeric result: 3 per step. */
MIDMAN_EXPORT int32_t midman_train_stage(uint32_t handle, const int32_t *inputs, const int32_t *targets);
MIDMAN_EXPORT int32_t midman_train_step_staged(uint32_t handle, uint32_t steps);
/* Loss and gradients without an update. Numeric result: [loss]. */
MIDMAN_EXPORT int32_t midman_train_loss_and_grads(uint32_t handle, const int32_t *inputs, const int32_t *targets);
/* Parameter values (which = 0), gradients (1), AdamW first (2) or second (3)
 * moments of tensor `index` in MidManModel::parameters order, or of the whole
 * flat vector when index == 0xFFFFFFFF. Numeric result: the values. */
MIDMAN_EXPORT int32_t midman_train_read(uint32_t handle, uint32_t which, uint32_t index);
/* midman_train_read with which = 0 (parameter values) and 1 (gradients): one
 * tensor D2H for parity checks, or the whole vector with index 0xFFFFFFFF. */
MIDMAN_EXPORT int32_t midman_train_params(uint32_t handle, uint32_t index);
MIDMAN_EXPORT int32_t midman_train_grads(uint32_t handle, uint32_t index);
/* Replaces every parameter (`len` must equal the parameter count). */
MIDMAN_EXPORT int32_t midman_train_load(uint32_t handle, const float *values, uint64_t len);
/* Text result: {"params":..,"steps":..,"kernel_launches":..,"tensors":[{"name":..,"shape":[..],"offset":..}]} */
MIDMAN_EXPORT int32_t midman_train_describe(uint32_t handle);
/* Forward only on batch x seq (<= the trainer's): numeric result [loss]. */
MIDMAN_EXPORT int32_t midman_train_eval(uint32_t handle, const int32_t *inputs, const int32_t *targets,
                                        uint32_t batch, uint32_t seq);
MIDMAN_EXPORT int32_t midman_train_destroy(uint32_t handle);
/* The cudaStream_t the trainer launches on (for callers that time with events). */
MIDMAN_EXPORT int32_t midman_train_stream(uint32_t handle, uint64_t *out);
/* enable != 0: bracket every GEMM and attention launch with CUDA events; totals
 * per kernel class appear under "profile" in midman_train_describe. */
MIDMAN_EXPORT int32_t midman_train_profile(uint32_t handle, uint32_t enable);

/* ---- batches (crates/midman-data/src/batch.rs:45-248): windows of seq + 1
 * tokens every seq tokens of one shard, visited in a per-epoch order from
 * Rng(seed).fork(epoch).shuffle. Returns a handle (>= 1) as the status. ---- */
MIDMAN_EXPORT int32_t midman_batcher_create(const uint32_t *tokens, uint64_t n, uint32_t vocab, uint32_t seq,
                                            uint32_t batch, uint32_t seed_lo, uint32_t seed_hi);
/* A shard of n ids uniform in [0, vocab) from Rng(token_seed).below (synthetic data). */
MIDMAN_EXPORT int32_t midman_batcher_synthetic(uint32_t token_seed, uint32_t vocab, uint64_t n, uint32_t seq,
                                               uint32_t batch, uint32_t seed_lo, uint32_t seed_hi);
/* Writes batch*seq inputs and targets. Text result: {"epoch":..,"index":..,"sequences":..}. */
MIDMAN_EXPORT int32_t midman_batcher_next(uint32_t handle, int32_t *inputs, int32_t *targets);
MIDMAN_EXPORT int32_t midman_batcher_destroy(uint32_t handle);

/* ---- Token shards (crates/midman-data/src/shard.rs) and the input pipeline.
 * A .mmtokens file: 32-byte header (MMTOKENS, version 1, token width 2 or 4,
 * vocabulary size, end-of-text id, u64 token count), little-endian ids, SHA-256
 * of everything before it. The readers refuse a file for the reasons of
 * TokenShard::from_bytes (shard.rs:137-219) with MIDMAN_ERR_OTHER. */

/* Text: {"vocab_size","eos","tokens","token_width"}. Needs no GPU. */
MIDMAN_EXPORT int32_t midman_shard_inspect(const uint8_t *path, uint32_t path_len);
/* TokenShard::load (shard.rs:255-262): as midman_shard_inspect, and the first
 * min(capacity, tokens) ids into `tokens`. */
MIDMAN_EXPORT int32_t midman_shard_read(const uint8_t *path, uint32_t path_len, uint32_t *tokens,
                                        uint64_t capacity);
/* TokenShard::new + save (shard.rs:59-82, :113-135, :221-253): the file of these
 * ids, written to `path`.tmp, synced, renamed over `path`. A vocabulary of 0, an
 * end-of-text id or an id not below the vocabulary is MIDMAN_ERR_ARGUMENT. */
MIDMAN_EXPORT int32_t midman_shard_write(const uint8_t *path, uint32_t path_len, uint32_t vocab_size,
                                         uint32_t eos, const uint32_t *tokens, uint64_t n);
/* SHA-256 (FIPS 180-4) of n bytes into digest[32] (crates/midman-data/src/hash.rs:
 * the checksum shards end with). */
MIDMAN_EXPORT int32_t midman_sha256(const uint8_t *data, uint64_t n, uint8_t *digest);
/* A batcher over the sequences of these shards (paths separated by '\n'),
 * Sequences::new + Batcher::new (batch.rs:38-70, :113-170): windows of seq+1
 * tokens that never cross from one shard to the next, all shards with one
 * vocabulary and end-of-text id. Returns the handle (> 0) or an error. */
MIDMAN_EXPORT int32_t midman_batcher_open(const uint8_t *paths, uint32_t paths_len, uint32_t seq, uint32_t batch,
                                          uint32_t seed_lo, uint32_t seed_hi);
/* Batcher::seek (batch.rs:191-210): the next batch is the one a continuous run
 * would take after batches_done batches of this epoch. Text: {"epoch",
 * "position","sequences"}. */
MIDMAN_EXPORT int32_t midman_batcher_seek(uint32_t handle, uint64_t epoch, uint64_t batches_done);
/* Trainer::step (trainer.rs:162-183) `steps` times with batches from the batcher,
 * which gives the global batch (batch * world rows of seq tokens); this rank
 * trains rows [rank * batch, (rank + 1) * batch). The host takes and prepares
 * the next batch (checks, pinned copy, embedding index) while the GPU runs the
 * current step; its ids cross to the device after that step. Floats:
 * [loss, grad_norm, lr] per completed step. A step that fails leaves the
 * weights, moments, step count and the batcher's place as they were
 * (MIDMAN_STOPPED). Text: {"epoch","position","sequences"} of the batcher. */
MIDMAN_EXPORT int32_t midman_train_run(uint32_t handle, uint32_t batcher, uint32_t steps);
/* Optimizer-state sharding (ZeRO stage 1; no counterpart in the reference, whose
 * trainer is one process). enable != 0: rank r keeps the AdamW moments of one
 * contiguous range of the flat parameter vector (1/world of them); each step
 * reduces every gradient bucket to its owners (ncclReduce) instead of
 * all-reducing it, takes the global norm from the ranks' shares of the fixed
 * sum-of-squares grid (the same number as unsharded), updates its own range and
 * broadcasts it, the next forward waiting bucket by bucket. The step's results
 * match the unsharded step's to rounding (NCCL's reduce and all-reduce may add in
 * other orders). While on: reading moments (midman_train_read 2/3) and
 * midman_train_save are collective (every rank calls them; rank 0 alone writes the
 * file); gradients after a step are whole only on the owner's range, so
 * midman_train_read 1 is refused until midman_train_loss_and_grads. enable == 0
 * gathers the moments back (collective). Text: {"sharding": {"optimizer",
 * "world","rank","ranges":[[begin,end]...],"buckets":[[begin,end]...]}}; the
 * same object appears in midman_train_describe. */
MIDMAN_EXPORT int32_t midman_train_shard_optimizer(uint32_t handle, uint32_t enable);
/* The plan optimizer sharding follows for a config and world size, without a GPU:
 * {"params","norm_block","norm_blocks","ranges":[[begin,end] per rank],
 * "buckets":[[begin,end]...]} (the ranges a trainer of that world reports). */
MIDMAN_EXPORT int32_t midman_shard_plan(const double *config, uint32_t world);
/* Trainer::evaluate (trainer.rs:209-262) over held-out shard files (paths
 * separated by '\n'), windows of the run's seq: batches of the run's global batch
 * (or all the sequences, if fewer), row k of the `rows` taken is sequence
 * k * len / rows, at most max_batches batches; no gradients, the weights are
 * untouched. Shards of another vocabulary than the model's, max_batches 0 or no
 * sequence: MIDMAN_ERR_ARGUMENT. Floats: [loss]; text {"loss","batches","tokens"}.
 * Under data parallelism every rank evaluates all rows (no collective). */
MIDMAN_EXPORT int32_t midman_train_evaluate(uint32_t handle, const uint8_t *paths, uint32_t paths_len,
                                            uint64_t max_batches);

/* ---- Training state files (crates/midman-training/src/state.rs:45-288 with the
 * safetensors container of crates/midman-checkpoint/src/safetensors.rs). A file
 * written here is the reference's state file: the same tensor names
 * (param/<name>, adamw.m/<name>, adamw.v/<name>), metadata (format,
 * state_version, step, epoch, position and the twelve train.* settings of
 * config.rs:113-131) and byte layout, so a GPU run resumes a CPU state and the
 * other way round. The data-order seed, epoch and position belong to the caller's
 * batcher; the global batch size is batch * world of midman_train_create. */

/* Writes <path>.tmp and renames it over path (safetensors.rs:224-253). */
MIDMAN_EXPORT int32_t midman_train_save(uint32_t handle, const uint8_t *path, uint32_t path_len,
                                        uint32_t data_seed_lo, uint32_t data_seed_hi, uint64_t epoch,
                                        uint64_t position);
/* Loads weights, both moments and the step count after every check of
 * load_state (state.rs:176-288) and AdamW::restore (adamw.rs:95-130); nothing
 * changes unless the whole load succeeds. Text: {"step","epoch","position"}.
 * Errors: MIDMAN_ERR_OTHER for a file that is not a valid state file (format,
 * version, header), MIDMAN_ERR_ARGUMENT for a state that does not fit the run
 * (settings, missing or extra tensors, bad moments), MIDMAN_ERR_SHAPE for a
 * tensor of another shape. */
MIDMAN_EXPORT int32_t midman_train_restore(uint32_t handle, const uint8_t *path, uint32_t path_len,
                                           uint32_t data_seed_lo, uint32_t data_seed_hi);
/* Reads and checks a safetensors file (TensorFile::from_bytes,
 * safetensors.rs:270-353; and progress_of, state.rs:125-173, when its format
 * entry says it is a training state) without a GPU. Text: {"metadata",
 * "tensors":[{"name","shape","data_offsets"}], "progress" (training states)}. */
MIDMAN_EXPORT int32_t midman_state_inspect(const uint8_t *path, uint32_t path_len);

#ifdef __cplusplus
}
#endif

#endif
