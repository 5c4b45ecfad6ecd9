// The device-resident training step: MidManModel forward, cross-entropy,
// backward, data-parallel gradient averaging, global-norm clip and AdamW
// (crates/midman-training/src/trainer.rs:185-207 and crates/midman-api/src/lab.rs:266-289),
// run as hand-written sm_100a kernels on one GPU per process.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <memory>
#include <string>
#include <vector>

#include "gemm.h"
#include "host.h"
#include "kernels.h"

namespace mm {

enum Precision : int { kPrecisionTF32 = 0, kPrecision3xTF32 = 1 };

struct StepOut {
  float loss = 0.0f;       // mean cross-entropy before the update (averaged over ranks)
  float grad_norm = 0.0f;  // global gradient norm before clipping
  bool ok = false;         // false: loss or norm not finite, nothing was changed
};

struct AdamHyper {
  float beta1 = 0.9f, beta2 = 0.95f, eps = 1e-8f, weight_decay = 0.1f, clip_norm = 1.0f;
};

class Trainer {
 public:
  // batch x seq is this rank's share of each step. world/rank/nccl_unique_id
  // (128 bytes) set up data parallelism; world == 1 needs none of them.
  Trainer(const ModelConfig& cfg, int batch, int seq, int precision, int world = 1, int rank = 0,
          const void* nccl_unique_id = nullptr);
  ~Trainer();
  Trainer(const Trainer&) = delete;
  Trainer& operator=(const Trainer&) = delete;

  const ModelConfig& config() const { return cfg_; }
  const ParamLayout& layout() const { return layout_; }
  int batch() const { return batch_; }
  int seq() const { return seq_; }
  int world() const { return world_; }
  int rank() const { return rank_; }
  uint64_t adam_steps() const { return adam_steps_; }
  cudaStream_t stream() const { return stream_; }

  // Seeded init on the host (reference draw order), copied to the device.
  void init_params(HostRng& rng, float init_std, int threads);
  void load_params(const float* host);
  void read_params(float* host);
  void read_grads(float* host);
  void read_moments(float* m, float* v);
  void read_tensor(uint64_t offset, uint64_t n, float* host, int which /*0 params, 1 grads, 2 m, 3 v*/);
  // Replaces parameters, both AdamW moments (null: zeros, for a run before its
  // first step) and the optimizer's step count, as a resumed run (state.rs:176-288).
  void restore(const float* params, const float* m, const float* v, uint64_t adam_steps);

  // One full step on host token ids (batch*seq each). lr from the caller's schedule.
  StepOut train_step(const int32_t* inputs, const int32_t* targets, float lr, const AdamHyper& h);
  // The same step split in two: stage_batch copies a batch to the device once,
  // step_staged then trains on the staged batch (inputs already in HBM).
  void stage_batch(const int32_t* inputs, const int32_t* targets);
  StepOut step_staged(float lr, const AdamHyper& h);
  // Forward + backward only: loss and gradients (averaged over ranks), no update.
  float loss_and_grads(const int32_t* inputs, const int32_t* targets);
  // Forward only on batch x seq (<= the capacity): mean loss, and the top-1
  // prediction per position when predictions != null.
  float eval(const int32_t* inputs, const int32_t* targets, int batch, int seq, int32_t* predictions);
  void logits(const int32_t* inputs, int batch, int seq, float* host_out);
  // Attention probabilities of every layer for batch x seq: [L, B, H, T, T].
  void attention_maps(const int32_t* inputs, int batch, int seq, float* host_out);
  // Per-tensor L2 norms of the last step's gradients (f64 accumulation).
  std::vector<float> grad_norms();

  // Optimizer-state sharding (ZeRO stage 1) over the data-parallel ranks. Rank r
  // keeps the AdamW moments of the flat range [shard_begin(r), shard_end(r)) only;
  // a step reduces each gradient bucket to the ranks owning it (ncclReduce, in
  // place of the all-reduce), takes the global norm from the ranks' shares of the
  // fixed sum-of-squares grid (one all-reduce of the partials, so it is the same
  // number as without sharding), updates its own range, and broadcasts it to the
  // others while the next step's forward waits layer by layer. The ranges end on
  // blocks of that grid. Turning it on keeps this rank's share of the moments;
  // turning it off gathers them (collective: every rank calls it).
  void shard_optimizer(bool on);
  bool optimizer_sharded() const { return zero1_; }
  uint64_t shard_begin(int r) const { return zero1_ ? bounds_[r] : 0; }
  uint64_t shard_end(int r) const { return zero1_ ? bounds_[r + 1] : layout_.total; }
  // The ranges of the flat vector the step reduces and broadcasts as one bucket,
  // in forward order: the embedding, each block, the final norm (and untied head).
  const std::vector<std::pair<uint64_t, uint64_t>>& buckets() const { return buckets_; }

  // Kernels this object launched since construction (counted by the launchers).
  uint64_t kernel_launches() const { return launches_; }

  // Per-kernel-class device timing: when on, every GEMM and attention launch is
  // bracketed by CUDA events on the trainer's stream; totals are collected when
  // each step synchronizes. flops are the algorithmic counts (2*M*N*K for a
  // GEMM; causal attention counts half of the T x T products).
  struct ProfileEntry {
    uint64_t launches = 0;
    double ms = 0.0, flops = 0.0;
  };
  void set_profile(bool on);
  const std::vector<std::pair<std::string, ProfileEntry>>& profile() const { return profile_; }
  // The GEMM class split by shape and operand majors ("MxNxK AB").
  const std::vector<std::pair<std::string, ProfileEntry>>& gemm_profile() const { return gemm_profile_; }

 private:
  void forward(int B, int T, bool train);
  void backward(int B, int T);
  void upload_batch(const int32_t* inputs, const int32_t* targets, int B, int T);
  StepOut finish_collect(bool update);
  void finish_launch(float lr, const AdamHyper& h, bool update);
  void build_embedding_csr(const int32_t* inputs, int N, int slot);
  // GEMMs on `st` (the trainer's stream when null). keep (3xTF32): no kernel has
  // written any operand since the previous product, whose lo copies may be reused.
  void gemm(int M, int N, int K, const float* A, long long lda, bool a_mn, const float* B, long long ldb, bool b_mn,
            float* C, long long ldc, const float* R, long long ldr, cudaStream_t st = nullptr, bool keep = false);
  void gemm_sum(int M, int N, const GemmSegment* segs, int nseg, float* C, long long ldc, const float* R,
                long long ldr, cudaStream_t st = nullptr, bool keep = false);
  StepOut finish_step(float lr, const AdamHyper& h, bool update);

 public:
  // The step split for a host that prepares the next batch while the GPU runs
  // this one: prepare_batch (host only: checks, pinned copy, embedding CSR) into
  // staging slot 0 or 1, upload_prepared (H2D on the step's stream), then
  // launch_step (no wait) and collect_step (waits, returns the results).
  void prepare_batch(const int32_t* inputs, const int32_t* targets, int B, int T, int slot);
  void upload_prepared(int slot, int B, int T, bool with_targets);
  void launch_step(float lr, const AdamHyper& h);
  StepOut collect_step();

 private:
  void allreduce_grads_range(uint64_t offset, uint64_t n);
  void reduce_bucket(int b);           // all-reduce, or reduce to the owners under sharding
  void broadcast_params();             // owners -> all, bucket by bucket (sharding)
  void wait_params(int bucket);        // stream_ waits for a bucket's broadcast (-1: all)
  void gather_moment(int which, uint64_t offset, uint64_t n, float* dst_device);
  void build_chunks();
  uint64_t mv_begin() const { return zero1_ ? bounds_[rank_] : 0; }
  void check_device(const char* where);
  void wait_exchange(const char* where);
  int prof_begin();
  void prof_end(int slot, const char* cls, double flops, std::string shape = {});
  void prof_collect();

  ModelConfig cfg_;
  ParamLayout layout_;
  int batch_, seq_, precision_, world_, rank_;
  uint64_t adam_steps_ = 0;
  uint64_t launches_ = 0;
  cudaStream_t stream_ = nullptr, comm_stream_ = nullptr;
  void* comm_ = nullptr;  // ncclComm_t; null after an abort
  // how long a step may wait for the exchange before the communicator is
  // aborted (MIDMAN_EXCHANGE_TIMEOUT_MS, default 10 minutes)
  long long exchange_timeout_ms_ = 600000;
  std::vector<cudaEvent_t> layer_done_;
  cudaEvent_t comm_done_ = nullptr;

  // parameters, gradients and AdamW moments, flat in parameter order (moments:
  // this rank's range only under optimizer sharding)
  float *P_ = nullptr, *G_ = nullptr, *M_ = nullptr, *V_ = nullptr;
  bool zero1_ = false;
  bool owner_reduce_ = false;   // this backward reduces to the owners (a sharded update)
  bool grads_partial_ = false;  // G_ is complete only on this rank's range
  std::vector<uint64_t> bounds_;                          // world + 1 range ends
  std::vector<std::pair<uint64_t, uint64_t>> buckets_;  // forward order
  std::vector<cudaEvent_t> gathered_;                   // per bucket: broadcast done
  bool gather_pending_ = false;
  cudaEvent_t update_done_ = nullptr;
  AdamChunk* d_chunks_ = nullptr;
  int n_chunks_ = 0;
  std::vector<std::pair<int, int>> bucket_chunks_;  // [first, end) chunk of each bucket (unsharded)
  float *d_cos_ = nullptr, *d_sin_ = nullptr;

  // token ids and the embedding-gradient CSR
  int32_t *d_ids_ = nullptr, *d_tgt_ = nullptr, *d_uniq_ = nullptr, *d_off_ = nullptr, *d_pos_ = nullptr;
  int n_uniq_ = 0;                            // distinct ids of the batch on the device
  int32_t* h_pinned_[2] = {nullptr, nullptr};  // two staging slots: ids, targets, uniq, offsets, positions
  int n_uniq_slot_[2] = {0, 0};
  std::vector<int32_t> h_ids_copy_;

  // saved activations, one set per layer
  struct Layer {
    float *x, *xn1, *rstd1, *q, *k, *v, *o, *lse, *h, *xn2, *rstd2, *g, *u, *act;
  };
  std::vector<Layer> acts_;
  float *x_final_ = nullptr, *xf_ = nullptr, *rstdf_ = nullptr, *logits_ = nullptr, *row_loss_ = nullptr;
  // backward scratch
  float *dx_[2] = {nullptr, nullptr}, *dxn_ = nullptr, *do_ = nullptr, *dq_ = nullptr, *dk_ = nullptr, *dv_ = nullptr,
        *dact_ = nullptr, *delta_ = nullptr, *norm_ws_ = nullptr, *tmp_ = nullptr;
  double *d_partials_ = nullptr, *d_loss_ = nullptr;
  float* d_norm_ = nullptr;  // [norm, clip factor, ok]
  int32_t* d_pred_ = nullptr;
  float* h_out_ = nullptr;   // pinned: loss (as 2 floats of a double), norm_out, error flag
  std::vector<void*> allocations_;
  int dx_cur_ = 0;  // which dx_ buffer holds the gradient flowing down

  // Attention on the tensor cores (TF32 mode, head_dim 32/64/128): score buffers.
  bool attn_tc_ = false;
  bool attn_3x_ = false;       // 3xTF32 attention on the tensor cores (score buffers in attn3_ws_)
  float* attn3_ws_ = nullptr;
  X3LoCache lo_cache_;  // 3xTF32 lo copies shared by consecutive products
  // The backward's side stream (weight-gradient products, the attention
  // backward's dQ kernel) and its events.
  cudaStream_t side_stream_ = nullptr;
  cudaEvent_t attn_side_ready_ = nullptr, attn_side_done_ = nullptr;
  cudaEvent_t side_ev_[4] = {nullptr, nullptr, nullptr, nullptr};

  bool profiling_ = false;
  std::vector<cudaEvent_t> prof_events_;
  struct Pending {
    int slot;
    std::string cls;
    double flops;
    std::string shape;  // GEMMs: "MxNxK AB" (A/B: K = K-major, M = MN-major)
  };
  std::vector<std::pair<std::string, ProfileEntry>> gemm_profile_;
  std::vector<Pending> pending_;
  int prof_next_ = 0;
  std::vector<std::pair<std::string, ProfileEntry>> profile_;
};

}  // namespace mm
