// Oracle part 1: Rng, ModelConfig, parameter layout, seeded init, rotary tables.
#include <algorithm>
// Test infrastructure only (see oracle.h).
#include <array>
#include <cmath>
#include <cstring>
#include <tuple>

#include "oracle_internal.h"

namespace orc {

// rng.rs:16-22
static uint64_t splitmix64(uint64_t& state) {
  state += 0x9E3779B97F4A7C15ull;
  uint64_t z = state;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

static inline uint64_t rotl(uint64_t x, int k) { return (x << k) | (x >> (64 - k)); }

// rng.rs:36-41
Rng::Rng(uint64_t seed) {
  uint64_t sm = seed;
  for (auto& w : s) w = splitmix64(sm);
}

// rng.rs:44-55
uint64_t Rng::next_u64() {
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

// rng.rs:58-60
float Rng::next_f32() { return static_cast<float>(next_u64() >> 40) * (1.0f / 16777216.0f); }
// rng.rs:63-65
double Rng::next_f64() { return static_cast<double>(next_u64() >> 11) * (1.0 / 9007199254740992.0); }
// rng.rs:68-70
float Rng::uniform(float lo, float hi) { return lo + (hi - lo) * next_f32(); }

// rng.rs:74-85 (Box-Muller with a cached second value; f64 ln/sin/cos from libm)
float Rng::normal() {
  if (has_spare) {
    has_spare = false;
    return spare;
  }
  const double u1 = 1.0 - next_f64();
  const double u2 = next_f64();
  const double radius = std::sqrt(-2.0 * std::log(u1));
  const double theta = 6.283185307179586 * u2;
  spare = static_cast<float>(radius * std::sin(theta));
  has_spare = true;
  return static_cast<float>(radius * std::cos(theta));
}

// rng.rs:92-106 (Lemire's nearly-divisionless method)
uint64_t Rng::below(uint64_t n) {
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

// rng.rs:118-120
Rng Rng::fork(uint64_t stream) { return Rng(next_u64() ^ (stream * 0x9E3779B97F4A7C15ull)); }

// crates/midman-api/src/ffi.rs:170-187 (the config array order)
Config config_from(const double* v) {
  Config c;
  c.vocab = static_cast<uint64_t>(v[0]);
  c.d_model = static_cast<uint64_t>(v[1]);
  c.n_layers = static_cast<uint64_t>(v[2]);
  c.n_heads = static_cast<uint64_t>(v[3]);
  c.n_kv_heads = static_cast<uint64_t>(v[4]);
  c.d_ff = static_cast<uint64_t>(v[5]);
  c.max_seq_len = static_cast<uint64_t>(v[6]);
  c.rope_theta = static_cast<float>(v[7]);
  c.norm_eps = static_cast<float>(v[8]);
  c.tie = v[9] != 0.0;
  return c;
}

// config.rs:106-137: the first invalid field, in the reference's order of checks.
std::string validate(const Config& c) {
  if (!c.vocab) return "vocab_size";
  if (!c.d_model) return "d_model";
  if (!c.n_layers) return "n_layers";
  if (!c.n_heads) return "n_heads";
  if (!c.n_kv_heads) return "n_kv_heads";
  if (!c.d_ff) return "d_ff";
  if (!c.max_seq_len) return "max_seq_len";
  if (!(std::isfinite(c.rope_theta) && c.rope_theta > 0.0f)) return "rope_theta";
  if (!(std::isfinite(c.norm_eps) && c.norm_eps > 0.0f)) return "norm_eps";
  if ((c.d_model / c.n_heads) * c.n_heads != c.d_model) return "n_heads";
  if ((c.n_heads / c.n_kv_heads) * c.n_kv_heads != c.n_heads) return "n_kv_heads";
  if (c.head_dim() & 1) return "d_model";
  return "";
}

// MidManModel::parameters order (model.rs:187-197; block.rs:85-91; attention.rs:248-255;
// mlp.rs:70-75) with the shapes Linear/Embedding/RmsNorm give their weights.
void build_layout(Model& m) {
  const Config& c = m.cfg;
  m.tensors.clear();
  m.blocks.clear();
  uint64_t off = 0;
  auto add = [&](const std::string& name, std::vector<uint64_t> shape) {
    ParamTensor t;
    t.name = name;
    t.shape = shape;
    t.offset = off;
    t.numel = 1;
    for (auto d : shape) t.numel *= d;
    off += t.numel;
    m.tensors.push_back(t);
    return t.offset;
  };
  const uint64_t d = c.d_model, kv = c.kv_dim(), ff = c.d_ff;
  m.embed = add("embed_tokens.weight", {c.vocab, d});
  for (uint64_t i = 0; i < c.n_layers; ++i) {
    const std::string p = "blocks." + std::to_string(i) + ".";
    BlockParams b;
    b.attn_norm = add(p + "attn_norm.weight", {d});
    b.q = add(p + "attn.q_proj.weight", {d, d});
    b.k = add(p + "attn.k_proj.weight", {d, kv});
    b.v = add(p + "attn.v_proj.weight", {d, kv});
    b.o = add(p + "attn.o_proj.weight", {d, d});
    b.mlp_norm = add(p + "mlp_norm.weight", {d});
    b.gate = add(p + "mlp.gate_proj.weight", {d, ff});
    b.up = add(p + "mlp.up_proj.weight", {d, ff});
    b.down = add(p + "mlp.down_proj.weight", {ff, d});
    m.blocks.push_back(b);
  }
  m.final_norm = add("final_norm.weight", {d});
  if (!c.tie) m.lm_head = add("lm_head.weight", {d, c.vocab});
  m.params.assign(off, 0.0f);
}

// MidManModel::with_init_std (model.rs:51-84): draws in construction order;
// Tensor::randn is std * normal() (tensor.rs:158-162); Init::scaled (init.rs:33-40).
void init_weights(Model& m, Rng& rng, float std_) {
  const Config& c = m.cfg;
  const float out_std = std_ / std::sqrt(2.0f * static_cast<float>(c.n_layers));
  const uint64_t d = c.d_model, kv = c.kv_dim(), ff = c.d_ff;
  // Drawn tensors in draw order (offset, count, std); norms are ones and draw nothing.
  std::vector<std::tuple<uint64_t, uint64_t, float>> runs;
  runs.emplace_back(m.embed, c.vocab * d, std_);
  for (const BlockParams& b : m.blocks) {
    for (uint64_t i = 0; i < d; ++i) m.params[b.attn_norm + i] = 1.0f;
    runs.emplace_back(b.q, d * d, std_);
    runs.emplace_back(b.k, d * kv, std_);
    runs.emplace_back(b.v, d * kv, std_);
    runs.emplace_back(b.o, d * d, out_std);
    for (uint64_t i = 0; i < d; ++i) m.params[b.mlp_norm + i] = 1.0f;
    runs.emplace_back(b.gate, d * ff, std_);
    runs.emplace_back(b.up, d * ff, std_);
    runs.emplace_back(b.down, ff * d, out_std);
  }
  for (uint64_t i = 0; i < d; ++i) m.params[m.final_norm + i] = 1.0f;
  if (!c.tie) runs.emplace_back(m.lm_head, d * c.vocab, std_);
  // Element e of the drawn stream is std * normal() for the e-th call. normal()
  // consumes two 64-bit draws per pair of values (rng.rs:74-85), so pair p starts
  // 2p draws after the stream start: walk the state once to find each chunk's
  // start, then evaluate the chunks' Box-Muller pairs on several threads.
  std::vector<uint64_t> where;  // flat element -> parameter offset, by run
  uint64_t total = 0;
  for (auto& r : runs) total += std::get<1>(r);
  std::vector<float> stream(total);
  uint64_t first = 0;
  if (total && rng.has_spare) {
    stream[0] = rng.spare;
    rng.has_spare = false;
    first = 1;
  }
  const uint64_t pairs = (total - first + 1) / 2;
  const uint64_t chunk = 1ull << 16;
  const uint64_t nchunks = (pairs + chunk - 1) / chunk;
  std::vector<std::array<uint64_t, 4>> starts(nchunks);
  for (uint64_t ch = 0; ch < nchunks; ++ch) {
    for (int w = 0; w < 4; ++w) starts[ch][w] = rng.s[w];
    const uint64_t np = std::min(chunk, pairs - ch * chunk);
    for (uint64_t k = 0; k < 2 * np; ++k) rng.next_u64();
  }
  float last_sin = 0.0f;
#pragma omp parallel for schedule(dynamic)
  for (long long ch = 0; ch < static_cast<long long>(nchunks); ++ch) {
    Rng local(0);
    for (int w = 0; w < 4; ++w) local.s[w] = starts[ch][w];
    const uint64_t p0 = ch * chunk, p1 = std::min(pairs, p0 + chunk);
    for (uint64_t p = p0; p < p1; ++p) {
      local.has_spare = false;
      const float cs = local.normal();  // draws two values, caches the sine part
      const uint64_t e = first + 2 * p;
      stream[e] = cs;
      if (e + 1 < total)
        stream[e + 1] = local.spare;
      else
        last_sin = local.spare;
    }
  }
  if ((total - first) & 1) {
    rng.spare = last_sin;
    rng.has_spare = true;
  }
  uint64_t pos = 0;
  for (auto& r : runs) {
    float* p = m.params.data() + std::get<0>(r);
    const float s = std::get<2>(r);
    for (uint64_t i = 0; i < std::get<1>(r); ++i) p[i] = s * stream[pos + i];
    pos += std::get<1>(r);
  }
  rope_tables(c.head_dim(), c.max_seq_len, c.rope_theta, m.rope_cos, m.rope_sin);
}

// RotaryTables::new (rope.rs:54-85): angles in f64, stored as f32.
void rope_tables(uint64_t head_dim, uint64_t max_seq_len, float theta, std::vector<float>& cos_out,
                 std::vector<float>& sin_out) {
  const uint64_t half = head_dim / 2;
  cos_out.resize(max_seq_len * half);
  sin_out.resize(max_seq_len * half);
  for (uint64_t pos = 0; pos < max_seq_len; ++pos) {
    for (uint64_t i = 0; i < half; ++i) {
      const double frequency = std::pow(static_cast<double>(theta), -static_cast<double>(i) / static_cast<double>(half));
      const double angle = static_cast<double>(pos) * frequency;
      cos_out[pos * half + i] = static_cast<float>(std::cos(angle));
      sin_out[pos * half + i] = static_cast<float>(std::sin(angle));
    }
  }
}

}  // namespace orc
