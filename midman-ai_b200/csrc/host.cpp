// Host-side configuration, parameter layout, seeded RNG, init and schedule.
#include "host.h"

#include <algorithm>
#include <array>
#include <cmath>
#include <stdexcept>
#include <thread>

namespace mm {

// ---------------------------------------------------------------- config
std::string validate_config(const ModelConfig& c) {
  // config.rs:106-137, same order of checks
  if (!c.vocab) return "vocab_size: must be greater than zero";
  if (!c.d_model) return "d_model: must be greater than zero";
  if (!c.n_layers) return "n_layers: must be greater than zero";
  if (!c.n_heads) return "n_heads: must be greater than zero";
  if (!c.n_kv_heads) return "n_kv_heads: must be greater than zero";
  if (!c.d_ff) return "d_ff: must be greater than zero";
  if (!c.max_seq_len) return "max_seq_len: must be greater than zero";
  if (!(std::isfinite(c.rope_theta) && c.rope_theta > 0.0f))
    return "rope_theta: must be a finite number greater than zero";
  if (!(std::isfinite(c.norm_eps) && c.norm_eps > 0.0f)) return "norm_eps: must be a finite number greater than zero";
  if ((c.d_model / c.n_heads) * c.n_heads != c.d_model)
    return "n_heads: d_model " + std::to_string(c.d_model) + " is not divisible by n_heads " + std::to_string(c.n_heads);
  if ((c.n_heads / c.n_kv_heads) * c.n_kv_heads != c.n_heads)
    return "n_kv_heads: n_heads " + std::to_string(c.n_heads) + " is not divisible by n_kv_heads " +
           std::to_string(c.n_kv_heads);
  if (c.head_dim() & 1)
    return "d_model: head dimension " + std::to_string(c.head_dim()) + " must be even for rotary embeddings";
  return "";
}

bool param_breakdown(const ModelConfig& c, ParamBreakdown* out, std::string* err) {
  const std::string bad = validate_config(c);
  if (!bad.empty()) {
    if (err) *err = bad;
    return false;
  }
  auto mul = [](uint64_t a, uint64_t b, uint64_t& r) { return !__builtin_mul_overflow(a, b, &r); };
  auto add = [](uint64_t a, uint64_t b, uint64_t& r) { return !__builtin_add_overflow(a, b, &r); };
  const uint64_t d = c.d_model, kv = c.kv_dim();
  uint64_t emb, t0, t1, t2, att, mlp, norms, total;
  bool ok = mul(c.vocab, d, emb) && mul(d, d, t0) && mul(2, t0, t0) && mul(d, kv, t1) && mul(2, t1, t1) &&
            add(t0, t1, t2) && mul(c.n_layers, t2, att) && mul(d, c.d_ff, t0) && mul(3, t0, t0) &&
            mul(c.n_layers, t0, mlp) && mul(2, d, t0) && mul(c.n_layers, t0, t0) && add(t0, d, norms);
  const uint64_t head = c.tie ? 0 : emb;
  ok = ok && add(emb, att, total) && add(total, mlp, total) && add(total, norms, total) && add(total, head, total);
  if (!ok) {
    if (err) *err = "model: parameter count overflows a 64-bit integer";
    return false;
  }
  *out = {emb, att, mlp, norms, head};
  return true;
}

const char* preset_name(int i) {
  static const char* names[kNumPresets] = {"smoke", "tiny", "small", "base", "medium", "large"};
  return (i >= 0 && i < kNumPresets) ? names[i] : nullptr;
}

ModelConfig preset_config(int i) {
  // (vocab, d_model, n_layers, n_heads, n_kv_heads, d_ff, max_seq_len)
  static const uint64_t p[kNumPresets][7] = {{256, 64, 2, 4, 4, 176, 128},          {4096, 128, 4, 4, 4, 344, 256},
                                             {32000, 384, 6, 6, 6, 1024, 512},      {32000, 768, 12, 12, 12, 2048, 1024},
                                             {32000, 1024, 24, 16, 8, 2816, 2048}, {32000, 2048, 20, 16, 8, 5632, 2048}};
  ModelConfig c;
  c.vocab = p[i][0];
  c.d_model = p[i][1];
  c.n_layers = p[i][2];
  c.n_heads = p[i][3];
  c.n_kv_heads = p[i][4];
  c.d_ff = p[i][5];
  c.max_seq_len = p[i][6];
  return c;
}

std::vector<std::pair<uint64_t, uint64_t>> gradient_buckets(const ModelConfig& c, const ParamLayout& L) {
  std::vector<std::pair<uint64_t, uint64_t>> b;
  b.push_back({L.embed, L.embed + c.vocab * c.d_model});
  for (const BlockOffsets& bo : L.blocks) b.push_back({bo.attn_norm, bo.down + c.d_ff * c.d_model});
  b.push_back({L.final_norm, L.total});
  return b;
}

std::vector<uint64_t> shard_bounds(uint64_t total, int world, uint64_t block, int blocks) {
  std::vector<uint64_t> bounds(world + 1, total);
  for (int r = 0; r < world; ++r)
    bounds[r] = std::min<uint64_t>(total, block * ((static_cast<uint64_t>(blocks) * r) / world));
  return bounds;
}

ParamLayout param_layout(const ModelConfig& c) {
  ParamLayout L;
  uint64_t off = 0;
  auto add = [&](std::string name, std::vector<uint64_t> shape) {
    TensorInfo t;
    t.name = std::move(name);
    t.shape = std::move(shape);
    t.offset = off;
    t.numel = 1;
    for (auto x : t.shape) t.numel *= x;
    off += t.numel;
    L.tensors.push_back(t);
    return t.offset;
  };
  const uint64_t d = c.d_model, kv = c.kv_dim(), ff = c.d_ff;
  L.embed = add("embed_tokens.weight", {c.vocab, d});
  for (uint64_t i = 0; i < c.n_layers; ++i) {
    const std::string p = "blocks." + std::to_string(i) + ".";
    BlockOffsets b;
    b.attn_norm = add(p + "attn_norm.weight", {d});
    b.q = add(p + "attn.q_proj.weight", {d, d});
    b.k = add(p + "attn.k_proj.weight", {d, kv});
    b.v = add(p + "attn.v_proj.weight", {d, kv});
    b.o = add(p + "attn.o_proj.weight", {d, d});
    b.mlp_norm = add(p + "mlp_norm.weight", {d});
    b.gate = add(p + "mlp.gate_proj.weight", {d, ff});
    b.up = add(p + "mlp.up_proj.weight", {d, ff});
    b.down = add(p + "mlp.down_proj.weight", {ff, d});
    L.blocks.push_back(b);
  }
  L.final_norm = add("final_norm.weight", {d});
  if (!c.tie) L.lm_head = add("lm_head.weight", {d, c.vocab});
  L.total = off;
  return L;
}

// ---------------------------------------------------------------- rng
namespace {
uint64_t splitmix64(uint64_t& x) {
  x += 0x9E3779B97F4A7C15ull;
  uint64_t z = x;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
inline uint64_t rotl(uint64_t x, int k) { return (x << k) | (x >> (64 - k)); }
inline uint64_t xoshiro_next(uint64_t* s) {
  const uint64_t result = rotl(s[1] * 5, 7) * 9;
  const uint64_t t = s[1] << 17;
  s[2] ^= s[0];
  s[3] ^= s[1];
  s[1] ^= s[2];
  s[0] ^= s[3];
  s[2] ^= t;
  s[3] = rotl(s[3], 45);
  return result;
}
inline double to_f64(uint64_t x) { return static_cast<double>(x >> 11) * (1.0 / 9007199254740992.0); }
// One Box-Muller pair from two draws (rng.rs:78-84): (cos part, sin part).
inline void box_muller(uint64_t a, uint64_t b, float* c, float* s) {
  const double u1 = 1.0 - to_f64(a);
  const double u2 = to_f64(b);
  const double radius = std::sqrt(-2.0 * std::log(u1));
  const double theta = 6.283185307179586 * u2;
  *s = static_cast<float>(radius * std::sin(theta));
  *c = static_cast<float>(radius * std::cos(theta));
}
}  // namespace

HostRng::HostRng(uint64_t seed) {
  uint64_t sm = seed;
  for (auto& w : s_) w = splitmix64(sm);
}
uint64_t HostRng::next_u64() { return xoshiro_next(s_); }
double HostRng::next_f64() { return to_f64(next_u64()); }
float HostRng::normal() {
  if (has_spare_) {
    has_spare_ = false;
    return spare_;
  }
  const uint64_t a = next_u64(), b = next_u64();
  float c, s;
  box_muller(a, b, &c, &s);
  spare_ = s;
  has_spare_ = true;
  return c;
}
uint64_t HostRng::below(uint64_t n) {
  unsigned __int128 product = static_cast<unsigned __int128>(next_u64()) * n;
  uint64_t low = static_cast<uint64_t>(product);
  if (low < n) {
    const uint64_t threshold = (0 - n) % n;
    while (low < threshold) {
      product = static_cast<unsigned __int128>(next_u64()) * n;
      low = static_cast<uint64_t>(product);
    }
  }
  return static_cast<uint64_t>(product >> 64);
}
HostRng HostRng::fork(uint64_t stream) { return HostRng(next_u64() ^ (stream * 0x9E3779B97F4A7C15ull)); }

void HostRng::normals_parallel(float* out, uint64_t n, const std::vector<std::pair<uint64_t, float>>& runs,
                               int threads) {
  // Scale of element i: the run that contains it.
  std::vector<uint64_t> run_end;
  std::vector<float> run_scale;
  uint64_t acc = 0;
  for (auto& r : runs) {
    acc += r.first;
    run_end.push_back(acc);
    run_scale.push_back(r.second);
  }
  auto scale_at = [&](uint64_t i, size_t& hint) {
    while (hint < run_end.size() && i >= run_end[hint]) ++hint;
    return run_scale[hint];
  };
  uint64_t i0 = 0;
  if (n && has_spare_) {
    size_t h = 0;
    out[0] = scale_at(0, h) * spare_;
    has_spare_ = false;
    i0 = 1;
  }
  const uint64_t rest = n - i0;
  const uint64_t pairs = (rest + 1) / 2;
  const uint64_t chunk = 1ull << 18;  // pairs per work item
  const uint64_t n_chunks = (pairs + chunk - 1) / chunk;
  std::vector<std::array<uint64_t, 4>> starts(n_chunks);
  for (uint64_t c = 0; c < n_chunks; ++c) {
    for (int w = 0; w < 4; ++w) starts[c][w] = s_[w];
    const uint64_t np = (c + 1 == n_chunks) ? pairs - c * chunk : chunk;
    for (uint64_t k = 0; k < 2 * np; ++k) xoshiro_next(s_);
  }
  float last_sin = 0.0f;
  auto work = [&](uint64_t c0, uint64_t c1) {
    size_t hint = 0;
    for (uint64_t c = c0; c < c1; ++c) {
      uint64_t st[4] = {starts[c][0], starts[c][1], starts[c][2], starts[c][3]};
      const uint64_t p0 = c * chunk, p1 = std::min(pairs, p0 + chunk);
      hint = 0;
      for (uint64_t p = p0; p < p1; ++p) {
        const uint64_t a = xoshiro_next(st), b = xoshiro_next(st);
        float cs, sn;
        box_muller(a, b, &cs, &sn);
        const uint64_t e = i0 + 2 * p;
        out[e] = scale_at(e, hint) * cs;
        if (e + 1 < n)
          out[e + 1] = scale_at(e + 1, hint) * sn;
        else
          last_sin = sn;
      }
    }
  };
  if (threads < 1) threads = 1;
  std::vector<std::thread> pool;
  const uint64_t per = (n_chunks + threads - 1) / threads;
  for (int t = 0; t < threads; ++t) {
    const uint64_t c0 = t * per, c1 = std::min(n_chunks, c0 + per);
    if (c0 < c1) pool.emplace_back(work, c0, c1);
  }
  for (auto& th : pool) th.join();
  if (rest & 1) {
    spare_ = last_sin;
    has_spare_ = true;
  }
}

void init_params(const ModelConfig& c, const ParamLayout& L, HostRng& rng, float std_, float* params, int threads) {
  // Init::scaled (crates/midman-nn/src/init.rs:33-40)
  const float out_std = std_ / std::sqrt(2.0f * static_cast<float>(c.n_layers));
  // Norm weights are ones and draw nothing; everything else is drawn in
  // parameter order, which is also the draw order (model.rs:56-72).
  std::vector<std::pair<uint64_t, float>> runs;
  std::vector<std::pair<uint64_t, uint64_t>> spans;  // (offset, numel) of drawn tensors
  uint64_t drawn = 0;
  for (const TensorInfo& t : L.tensors) {
    if (t.shape.size() == 1) {
      for (uint64_t i = 0; i < t.numel; ++i) params[t.offset + i] = 1.0f;
      continue;
    }
    const bool residual = t.name.find("o_proj") != std::string::npos || t.name.find("down_proj") != std::string::npos;
    runs.push_back({t.numel, residual ? out_std : std_});
    spans.push_back({t.offset, t.numel});
    drawn += t.numel;
  }
  // Drawn tensors are not contiguous (norm weights sit between them): generate
  // into a staging buffer and scatter.
  std::vector<float> stage(drawn);
  rng.normals_parallel(stage.data(), drawn, runs, threads);
  uint64_t pos = 0;
  for (auto& sp : spans) {
    std::copy(stage.begin() + pos, stage.begin() + pos + sp.second, params + sp.first);
    pos += sp.second;
  }
}

void rope_tables(uint64_t head_dim, uint64_t max_seq_len, float theta, std::vector<float>& cos_out,
                 std::vector<float>& sin_out) {
  const uint64_t half = head_dim / 2;
  cos_out.resize(max_seq_len * half);
  sin_out.resize(max_seq_len * half);
  for (uint64_t pos = 0; pos < max_seq_len; ++pos)
    for (uint64_t i = 0; i < half; ++i) {
      const double freq = std::pow(static_cast<double>(theta), -static_cast<double>(i) / static_cast<double>(half));
      const double angle = static_cast<double>(pos) * freq;
      cos_out[pos * half + i] = static_cast<float>(std::cos(angle));
      sin_out[pos * half + i] = static_cast<float>(std::sin(angle));
    }
}

Batcher::Batcher(std::vector<uint32_t> tokens, uint32_t vocab, int seq, int batch, uint64_t seed)
    : Batcher(std::vector<std::vector<uint32_t>>{std::move(tokens)}, vocab, seq, batch, seed) {}

Sequences::Sequences(std::vector<std::vector<uint32_t>> shards, int seq) : shards_(std::move(shards)), seq_(seq) {
  if (seq <= 0) throw std::invalid_argument("a sequence must have at least one token");
  size_t total = 0;
  for (const auto& shard : shards_) {
    if (shard.size() > seq_) total += (shard.size() - 1) / seq_;  // batch.rs:63-67
    ends_.push_back(total);
  }
}

const uint32_t* Sequences::window(uint64_t index) const {
  // the first shard whose running count passes `index`
  const size_t shard = std::upper_bound(ends_.begin(), ends_.end(), static_cast<size_t>(index)) - ends_.begin();
  const size_t before = shard == 0 ? 0 : ends_[shard - 1];
  return shards_[shard].data() + (index - before) * seq_;
}

Batcher::Batcher(std::vector<std::vector<uint32_t>> shards, uint32_t vocab, int seq, int batch, uint64_t seed)
    : data_(std::move(shards), seq), vocab_(vocab), seq_(seq), batch_(batch), seed_(seed) {
  if (batch <= 0) throw std::invalid_argument("a batch must have at least one sequence");
  for (const auto& shard : data_.shards())
    for (uint32_t t : shard)
      if (t >= vocab_) throw std::out_of_range("token id " + std::to_string(t) + " is out of range for vocab " +
                                               std::to_string(vocab_));
  count_ = data_.size();
  if (count_ < batch_)
    throw std::invalid_argument("there are " + std::to_string(count_) + " sequences, fewer than one batch of " +
                                std::to_string(batch_));
  permute();
}

// batch.rs:244-248: Rng(seed).fork(epoch).shuffle(0..n)
void Batcher::permute() {
  order_.resize(count_);
  for (size_t i = 0; i < count_; ++i) order_[i] = i;
  HostRng r(seed_);
  HostRng f = r.fork(epoch_);
  f.shuffle(order_);
}

// batch.rs:213-240
std::pair<uint64_t, uint64_t> Batcher::next(int32_t* inputs, int32_t* targets) {
  if (next_ == batches_per_epoch()) {
    epoch_ += 1;
    next_ = 0;
    permute();
  }
  for (size_t r = 0; r < batch_; ++r) {
    const uint32_t* w = data_.window(order_[next_ * batch_ + r]);
    for (size_t t = 0; t < seq_; ++t) {
      inputs[r * seq_ + t] = static_cast<int32_t>(w[t]);
      targets[r * seq_ + t] = static_cast<int32_t>(w[t + 1]);
    }
  }
  const std::pair<uint64_t, uint64_t> at{epoch_, next_};
  next_ += 1;
  return at;
}

// batch.rs:197-210
void Batcher::seek(uint64_t epoch, uint64_t done) {
  if (done > batches_per_epoch())
    throw std::invalid_argument(std::to_string(done) + " batches done is more than the " +
                                std::to_string(batches_per_epoch()) + " in a pass");
  if (epoch != epoch_) {
    epoch_ = epoch;
    permute();
  }
  next_ = done;
}

std::vector<uint32_t> synthetic_tokens(uint64_t seed, uint32_t vocab, uint64_t n) {
  HostRng r(seed);
  std::vector<uint32_t> out(n);
  for (auto& t : out) t = static_cast<uint32_t>(r.below(vocab));
  return out;
}

float schedule_lr(float max_lr, float min_lr, uint64_t warmup, uint64_t total, uint64_t step) {
  const double mx = max_lr, mn = min_lr;
  if (step < warmup) return static_cast<float>(mx * static_cast<double>(step + 1) / static_cast<double>(warmup));
  if (step >= total) return min_lr;
  const double progress = static_cast<double>(step - warmup) / static_cast<double>(total - warmup);
  return static_cast<float>(mn + 0.5 * (mx - mn) * (1.0 + std::cos(3.141592653589793 * progress)));
}

}  // namespace mm
