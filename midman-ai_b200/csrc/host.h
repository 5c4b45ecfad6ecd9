// Host-side pieces of the training step that the device kernels need as
// inputs: the model configuration and its parameter layout, the seeded random
// number generator, the learning-rate schedule and the batcher.
#pragma once
#include <cstdint>
#include <string>
#include <vector>

namespace mm {

// crates/midman-model-config/src/config.rs:19-42
struct ModelConfig {
  uint64_t vocab = 0, d_model = 0, n_layers = 0, n_heads = 0, n_kv_heads = 0, d_ff = 0, max_seq_len = 0;
  float rope_theta = 10000.0f, norm_eps = 1e-5f;
  bool tie = true;
  uint64_t head_dim() const { return d_model / n_heads; }
  uint64_t kv_dim() const { return n_kv_heads * head_dim(); }
};

// Validation in the reference's order of checks (config.rs:106-137). Returns an
// empty string when valid, otherwise "field: reason".
std::string validate_config(const ModelConfig& c);

struct ParamBreakdown {
  uint64_t embedding, attention, mlp, norms, lm_head;
  uint64_t total() const { return embedding + attention + mlp + norms + lm_head; }
};
// config.rs:158-183 with overflow checks; false + message on error.
bool param_breakdown(const ModelConfig& c, ParamBreakdown* out, std::string* err);

// The presets (crates/midman-model-config/src/presets.rs:61-83), smallest first.
constexpr int kNumPresets = 6;
const char* preset_name(int index);
ModelConfig preset_config(int index);

struct TensorInfo {
  std::string name;
  std::vector<uint64_t> shape;
  uint64_t offset = 0, numel = 0;
};
struct BlockOffsets {
  uint64_t attn_norm, q, k, v, o, mlp_norm, gate, up, down;
};
// The flat parameter vector in MidManModel::parameters order (model.rs:187-197),
// each tensor in the reference's own row-major layout ([in, out] for linears).
struct ParamLayout {
  std::vector<TensorInfo> tensors;
  std::vector<BlockOffsets> blocks;
  uint64_t embed = 0, final_norm = 0, lm_head = 0, total = 0;
};
ParamLayout param_layout(const ModelConfig& c);

// The flat ranges a data-parallel step exchanges as one bucket, in forward order:
// the embedding, each block, the final norm (and an untied head).
std::vector<std::pair<uint64_t, uint64_t>> gradient_buckets(const ModelConfig& c, const ParamLayout& L);
// Optimizer sharding: rank r owns [bounds[r], bounds[r + 1]) of the flat vector.
// The bounds are multiples of `block` elements (the gradient norm's fixed grid
// block), about total / world apart.
std::vector<uint64_t> shard_bounds(uint64_t total, int world, uint64_t block, int blocks);

// crates/midman-foundation/src/rng.rs:16-119 (xoshiro256** seeded by SplitMix64,
// Box-Muller normals with a cached second value).
class HostRng {
 public:
  explicit HostRng(uint64_t seed);
  uint64_t next_u64();
  double next_f64();
  float normal();
  uint64_t below(uint64_t n);
  HostRng fork(uint64_t stream);
  template <class T>
  void shuffle(std::vector<T>& v) {
    for (size_t i = v.size(); i-- > 1;) std::swap(v[i], v[static_cast<size_t>(below(i + 1))]);
  }
  // Fills out[i] = scale_of(i) * normal() for i in [0, n) exactly as n calls
  // would, using `threads` threads: one pass advances the state and records
  // where each chunk starts, then the chunks' Box-Muller transforms run in
  // parallel. Leaves the generator as n sequential calls would.
  void normals_parallel(float* out, uint64_t n, const std::vector<std::pair<uint64_t, float>>& scale_runs,
                        int threads);

 private:
  uint64_t s_[4];
  bool has_spare_ = false;
  float spare_ = 0.0f;
};

// MidManModel::with_init_std (model.rs:51-84): draws every weight in order.
void init_params(const ModelConfig& c, const ParamLayout& layout, HostRng& rng, float std_, float* params,
                 int threads);

// RotaryTables::new (crates/midman-nn/src/rope.rs:54-85): angles in f64.
void rope_tables(uint64_t head_dim, uint64_t max_seq_len, float theta, std::vector<float>& cos_out,
                 std::vector<float>& sin_out);

// Sequences over one token shard (windows of seq + 1 tokens every seq tokens)
// and the seeded Batcher (crates/midman-data/src/batch.rs:45-248).
// Sequences (batch.rs:29-107): windows of seq + 1 tokens every seq tokens of each
// shard; a window never crosses from one shard to the next.
class Sequences {
 public:
  Sequences(std::vector<std::vector<uint32_t>> shards, int seq);
  size_t size() const { return ends_.empty() ? 0 : ends_.back(); }
  size_t seq() const { return seq_; }
  const std::vector<std::vector<uint32_t>>& shards() const { return shards_; }
  const uint32_t* window(uint64_t index) const;  // Sequences::window (batch.rs:96-106); index < size()

 private:
  std::vector<std::vector<uint32_t>> shards_;
  std::vector<size_t> ends_;  // sequences in each shard and all the shards before it
  size_t seq_;
};

class Batcher {
 public:
  Batcher(std::vector<uint32_t> tokens, uint32_t vocab, int seq, int batch, uint64_t seed);
  // Sequences::new (batch.rs:38-70) over several shards: windows never cross
  // from one shard to the next.
  Batcher(std::vector<std::vector<uint32_t>> shards, uint32_t vocab, int seq, int batch, uint64_t seed);
  size_t sequences() const { return count_; }
  size_t batches_per_epoch() const { return count_ / batch_; }
  size_t batch() const { return batch_; }
  size_t seq() const { return seq_; }
  uint64_t epoch() const { return epoch_; }
  size_t position() const { return next_; }  // batches of the epoch handed out (batch.rs:186-189)
  // Writes batch * seq inputs and targets (int32). Returns (epoch, index) of the batch.
  std::pair<uint64_t, uint64_t> next(int32_t* inputs, int32_t* targets);
  void seek(uint64_t epoch, uint64_t done);

 private:
  void permute();
  Sequences data_;
  uint32_t vocab_;
  size_t seq_, batch_, count_;
  uint64_t seed_, epoch_ = 0;
  size_t next_ = 0;
  std::vector<uint64_t> order_;
};

// n token ids uniform in [0, vocab) from Rng(seed).below (the synthetic shard).
std::vector<uint32_t> synthetic_tokens(uint64_t seed, uint32_t vocab, uint64_t n);

// WarmupCosine::lr (crates/midman-optim/src/schedule.rs:54-64).
float schedule_lr(float max_lr, float min_lr, uint64_t warmup, uint64_t total, uint64_t step);

}  // namespace mm
