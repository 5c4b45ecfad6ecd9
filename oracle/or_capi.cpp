// Oracle part 4: optimizer, schedule, batcher and the C ABI of oracle.h.
// Test infrastructure only (see oracle.h).
#include <cmath>
#include <cstring>
#include <string>
#include <vector>

#include "oracle.h"
#include "oracle_internal.h"

using namespace orc;

namespace {

struct AdamW {
  float beta1, beta2, eps, wd;
  uint64_t steps = 0;
  std::vector<float> m, v;
  std::vector<char> decay;  // per element: parameter has rank >= 2 (adamw.rs:197)
};

// Sequences over shards + Batcher (crates/midman-data/src/batch.rs:38-248).
struct Batcher {
  std::vector<uint32_t> tokens;  // the shards one after another
  std::vector<size_t> starts;    // where each shard begins in `tokens`
  std::vector<size_t> ends;      // sequences in each shard and the ones before (batch.rs:61-68)
  size_t seq, batch, count;
  uint64_t seed, epoch = 0;
  size_t next = 0;
  std::vector<uint64_t> order;
  void permute() {  // batch.rs:244-248
    order.resize(count);
    for (size_t i = 0; i < count; ++i) order[i] = i;
    Rng r(seed);
    Rng f = r.fork(epoch);
    f.shuffle(order);
  }
  const uint32_t* window(size_t index) const {  // batch.rs:96-106
    size_t shard = 0;
    while (ends[shard] <= index) ++shard;
    const size_t before = shard == 0 ? 0 : ends[shard - 1];
    return tokens.data() + starts[shard] + (index - before) * seq;
  }
};

}  // namespace

extern "C" {

void or_set_threads(int n) { set_threads(n); }

void* or_rng_new(uint64_t seed) { return new Rng(seed); }
void or_rng_free(void* r) { delete static_cast<Rng*>(r); }
uint64_t or_rng_next_u64(void* r) { return static_cast<Rng*>(r)->next_u64(); }
float or_rng_next_f32(void* r) { return static_cast<Rng*>(r)->next_f32(); }
double or_rng_next_f64(void* r) { return static_cast<Rng*>(r)->next_f64(); }
float or_rng_uniform(void* r, float lo, float hi) { return static_cast<Rng*>(r)->uniform(lo, hi); }
float or_rng_normal(void* r) { return static_cast<Rng*>(r)->normal(); }
uint64_t or_rng_below(void* r, uint64_t n) { return n ? static_cast<Rng*>(r)->below(n) : 0; }
void or_rng_shuffle(void* r, uint64_t* items, size_t n) {
  std::vector<uint64_t> v(items, items + n);
  static_cast<Rng*>(r)->shuffle(v);
  std::memcpy(items, v.data(), n * sizeof(uint64_t));
}
void* or_rng_fork(void* r, uint64_t stream) { return new Rng(static_cast<Rng*>(r)->fork(stream)); }

// config.rs:158-183 (checked arithmetic: an overflow is a config error)
int or_param_breakdown(const double* cfg, uint64_t* out, char* msg, size_t cap) {
  const Config c = config_from(cfg);
  std::string bad = validate(c);
  auto mul = [&](uint64_t a, uint64_t b, uint64_t& r) { return !__builtin_mul_overflow(a, b, &r); };
  auto add = [&](uint64_t a, uint64_t b, uint64_t& r) { return !__builtin_add_overflow(a, b, &r); };
  uint64_t emb = 0, att = 0, mlp = 0, norms = 0, head = 0, t0, t1, t2, total;
  bool ok = bad.empty();
  const uint64_t d = c.d_model, kv = ok ? c.kv_dim() : 0;
  ok = ok && mul(c.vocab, d, emb);
  ok = ok && mul(d, d, t0) && mul(2, t0, t0) && mul(d, kv, t1) && mul(2, t1, t1) && add(t0, t1, t2) &&
       mul(c.n_layers, t2, att);
  ok = ok && mul(d, c.d_ff, t0) && mul(3, t0, t0) && mul(c.n_layers, t0, mlp);
  ok = ok && mul(2, d, t0) && mul(c.n_layers, t0, t0) && add(t0, d, norms);
  head = c.tie ? 0 : emb;
  ok = ok && add(emb, att, total) && add(total, mlp, total) && add(total, norms, total) && add(total, head, total);
  if (!ok) {
    if (bad.empty()) bad = "model";
    if (msg && cap) {
      std::strncpy(msg, bad.c_str(), cap - 1);
      msg[cap - 1] = 0;
    }
    return -2;
  }
  out[0] = emb;
  out[1] = att;
  out[2] = mlp;
  out[3] = norms;
  out[4] = head;
  out[5] = total;
  return 0;
}

int or_rope_table(int head_dim, int max_seq_len, float theta, float* cos_out, float* sin_out) {
  if (head_dim <= 0 || (head_dim & 1) || max_seq_len <= 0 || !(std::isfinite(theta) && theta > 0)) return -1;
  std::vector<float> c, s;
  rope_tables(head_dim, max_seq_len, theta, c, s);
  std::memcpy(cos_out, c.data(), c.size() * sizeof(float));
  std::memcpy(sin_out, s.data(), s.size() * sizeof(float));
  return 0;
}

void* or_model_new(const double* cfg, void* rng, float init_std) {
  Model* m = new Model;
  m->cfg = config_from(cfg);
  if (!validate(m->cfg).empty()) {
    delete m;
    return nullptr;
  }
  build_layout(*m);
  init_weights(*m, *static_cast<Rng*>(rng), init_std);
  return m;
}
void or_model_free(void* m) { delete static_cast<Model*>(m); }
size_t or_model_num_params(void* m) { return static_cast<Model*>(m)->params.size(); }
int or_model_num_tensors(void* m) { return static_cast<int>(static_cast<Model*>(m)->tensors.size()); }
int or_model_param_info(void* mp, int i, char* name, size_t cap, int* rank, int64_t* shape, uint64_t* offset,
                        uint64_t* numel) {
  Model* m = static_cast<Model*>(mp);
  if (i < 0 || i >= static_cast<int>(m->tensors.size())) return -1;
  const ParamTensor& t = m->tensors[i];
  if (name && cap) {
    std::strncpy(name, t.name.c_str(), cap - 1);
    name[cap - 1] = 0;
  }
  *rank = static_cast<int>(t.shape.size());
  for (size_t k = 0; k < t.shape.size(); ++k) shape[k] = static_cast<int64_t>(t.shape[k]);
  *offset = t.offset;
  *numel = t.numel;
  return 0;
}
void or_model_get_params(void* m, float* out) {
  auto& p = static_cast<Model*>(m)->params;
  std::memcpy(out, p.data(), p.size() * sizeof(float));
}
void or_model_set_params(void* m, const float* in) {
  auto& p = static_cast<Model*>(m)->params;
  std::memcpy(p.data(), in, p.size() * sizeof(float));
}
int or_model_loss(void* m, const int32_t* inputs, const int32_t* targets, int batch, int seq, float* loss,
                  float* grads) {
  return model_loss(*static_cast<Model*>(m), inputs, targets, batch, seq, loss, grads, nullptr, nullptr);
}
int or_model_logits(void* mp, const int32_t* inputs, int batch, int seq, float* logits) {
  std::vector<float> out;
  int rc = model_loss(*static_cast<Model*>(mp), inputs, nullptr, batch, seq, nullptr, nullptr, &out, nullptr);
  if (rc == 0) std::memcpy(logits, out.data(), out.size() * sizeof(float));
  return rc;
}
int or_model_attention(void* mp, const int32_t* inputs, int batch, int seq, float* probs) {
  std::vector<float> out;
  int rc = model_loss(*static_cast<Model*>(mp), inputs, nullptr, batch, seq, nullptr, nullptr, nullptr, &out);
  if (rc == 0) std::memcpy(probs, out.data(), out.size() * sizeof(float));
  return rc;
}

// clip.rs:29-59
float or_clip_global_norm(float* grads, size_t n, float max_norm, int* ok) {
  double sum = 0.0;
  for (size_t i = 0; i < n; ++i) sum += static_cast<double>(grads[i]) * static_cast<double>(grads[i]);
  const float norm = static_cast<float>(std::sqrt(sum));
  if (!std::isfinite(norm)) {
    *ok = 0;
    return norm;
  }
  *ok = 1;
  if (norm > max_norm) {
    const float factor = max_norm / (norm + 1e-6f);
    for (size_t i = 0; i < n; ++i) grads[i] *= factor;
  }
  return norm;
}

// schedule.rs:54-64
float or_schedule_lr(float max_lr, float min_lr, uint64_t warmup, uint64_t total, uint64_t step) {
  const double mx = max_lr, mn = min_lr;
  if (step < warmup) return static_cast<float>(mx * static_cast<double>(step + 1) / static_cast<double>(warmup));
  if (step >= total) return min_lr;
  const double progress = static_cast<double>(step - warmup) / static_cast<double>(total - warmup);
  return static_cast<float>(mn + 0.5 * (mx - mn) * (1.0 + std::cos(3.141592653589793 * progress)));
}

void* or_adamw_new(void* mp, float beta1, float beta2, float eps, float weight_decay) {
  Model* m = static_cast<Model*>(mp);
  AdamW* o = new AdamW{beta1, beta2, eps, weight_decay};
  o->m.assign(m->params.size(), 0.0f);
  o->v.assign(m->params.size(), 0.0f);
  o->decay.assign(m->params.size(), 0);
  for (const ParamTensor& t : m->tensors)
    if (t.shape.size() >= 2) std::memset(o->decay.data() + t.offset, 1, t.numel);
  return o;
}
void or_adamw_free(void* o) { delete static_cast<AdamW*>(o); }
uint64_t or_adamw_steps(void* o) { return static_cast<AdamW*>(o)->steps; }
void or_adamw_moments(void* op, float* m, float* v) {
  AdamW* o = static_cast<AdamW*>(op);
  std::memcpy(m, o->m.data(), o->m.size() * sizeof(float));
  std::memcpy(v, o->v.data(), o->v.size() * sizeof(float));
}
// AdamW::restore (adamw.rs:95-130) for the whole flat vector: steps and both
// moments; refuses non-finite m and negative or non-finite v (returns -1).
int or_adamw_restore(void* op, uint64_t steps, const float* m, const float* v) {
  AdamW* o = static_cast<AdamW*>(op);
  for (size_t i = 0; i < o->m.size(); ++i)
    if (!std::isfinite(m[i]) || !std::isfinite(v[i]) || v[i] < 0.0f) return -1;
  std::memcpy(o->m.data(), m, o->m.size() * sizeof(float));
  std::memcpy(o->v.data(), v, o->v.size() * sizeof(float));
  o->steps = steps;
  return 0;
}

}  // extern "C"

namespace orc {
void adamw_update(float* x, const float* g, float* m, float* v, size_t n, bool decay_on, uint64_t step, float lr,
                  float beta1, float beta2, float eps, float weight_decay) {
  const double t = static_cast<double>(step);
  const float bias1 = static_cast<float>(1.0 - std::pow(static_cast<double>(beta1), t));
  const float bias2_sqrt = static_cast<float>(std::sqrt(1.0 - std::pow(static_cast<double>(beta2), t)));
  const float step_size = lr / bias1;
  const float decay = decay_on ? 1.0f - lr * weight_decay : 1.0f;
#pragma omp parallel for schedule(static) if (n > (1u << 16))
  for (long long i = 0; i < static_cast<long long>(n); ++i) {
    x[i] *= decay;
    m[i] = beta1 * m[i] + (1.0f - beta1) * g[i];
    v[i] = beta2 * v[i] + (1.0f - beta2) * g[i] * g[i];
    x[i] -= step_size * m[i] / (std::sqrt(v[i]) / bias2_sqrt + eps);
  }
}
}  // namespace orc

extern "C" {

// adamw.rs:141-217 (validated first: a non-finite gradient or lr changes nothing)
int or_adamw_step(void* op, void* mp, const float* g, float lr) {
  AdamW* o = static_cast<AdamW*>(op);
  Model* m = static_cast<Model*>(mp);
  const size_t n = m->params.size();
  if (!(std::isfinite(lr) && lr >= 0.0f)) return -1;
  for (size_t i = 0; i < n; ++i)
    if (!std::isfinite(g[i])) return -1;
  o->steps += 1;
  for (const ParamTensor& t : m->tensors)
    adamw_update(m->params.data() + t.offset, g + t.offset, o->m.data() + t.offset, o->v.data() + t.offset,
                 t.numel, t.shape.size() >= 2, o->steps, lr, o->beta1, o->beta2, o->eps, o->wd);
  return 0;
}

int or_adamw_update(float* x, const float* g, float* m, float* v, size_t n, int decay, uint64_t step, float lr,
                    float beta1, float beta2, float eps, float weight_decay) {
  adamw_update(x, g, m, v, n, decay != 0, step, lr, beta1, beta2, eps, weight_decay);
  return 0;
}

void or_gemm_nn(const float* a, const float* b, float* c, size_t m, size_t k, size_t n) { gemm_nn(a, b, c, m, k, n); }
void or_gemm_nt(const float* a, const float* b, float* c, size_t m, size_t k, size_t n) { gemm_nt(a, b, c, m, k, n); }
void or_gemm_tn(const float* a, const float* b, float* c, size_t k, size_t m, size_t n) { gemm_tn(a, b, c, k, m, n); }
void or_softmax_rows(const float* x, float* y, size_t rows, size_t cols) { softmax_rows(x, y, rows, cols); }
void or_rms_norm(const float* x, const float* w, size_t rows, size_t d, float eps, float* y, float* rstd) {
  rms_norm_layer(x, w, rows, d, eps, y, rstd);
}
void or_rms_norm_bwd(const float* x, const float* w, const float* gy, size_t rows, size_t d, float eps, float* dx,
                     float* dw) {
  rms_norm_layer_bwd(x, w, gy, rows, d, eps, dx, dw);
}
void or_rope(float* x, size_t bh, size_t t, size_t hd, const float* cos_t, const float* sin_t, int backward) {
  rope_layer(x, bh, t, hd, cos_t, sin_t, backward != 0);
}
void or_swiglu(const float* g, const float* u, size_t n, float* act, const float* dact, float* dg, float* du) {
  swiglu_layer(g, u, n, act, dact, dg, du);
}
void or_embedding(const int32_t* ids, size_t rows, const float* table, size_t d, float* out, const float* dx,
                  float* dtable) {
  embedding_layer(ids, rows, table, d, out, dx, dtable);
}
float or_cross_entropy(const float* logits, const int32_t* targets, size_t n, size_t v, float* grad) {
  return cross_entropy(logits, targets, n, v, grad);
}
int or_causal_attention(const double* cfg, const float* q, const float* k, const float* v, int batch, int seq,
                        float* out, float* probs) {
  const Config c = config_from(cfg);
  if (!validate(c).empty()) return -2;
  causal_attention(c, q, k, v, batch, seq, out, probs);
  return 0;
}

// Trainer::update (trainer.rs:185-207)
int or_train_update(void* mp, void* op, const int32_t* inputs, const int32_t* targets, int batch, int seq,
                    float clip_norm, float lr, float* out) {
  Model* m = static_cast<Model*>(mp);
  std::vector<float> grads(m->params.size());
  float loss = 0.0f;
  int rc = model_loss(*m, inputs, targets, batch, seq, &loss, grads.data(), nullptr, nullptr);
  if (rc) return rc;
  out[0] = loss;
  if (!std::isfinite(loss)) return -1;
  int ok = 0;
  out[1] = or_clip_global_norm(grads.data(), grads.size(), clip_norm, &ok);
  if (!ok) return -1;
  return or_adamw_step(op, mp, grads.data(), lr);
}

void* or_batcher_new_shards(const uint32_t* tokens, const size_t* lens, size_t n_shards, int seq, int batch,
                            uint64_t seed) {
  if (seq <= 0 || batch <= 0) return nullptr;
  Batcher* b = new Batcher;
  b->seq = seq;
  b->batch = batch;
  b->count = 0;
  size_t at = 0;
  for (size_t i = 0; i < n_shards; ++i) {
    b->starts.push_back(at);
    b->tokens.insert(b->tokens.end(), tokens + at, tokens + at + lens[i]);
    if (lens[i] > static_cast<size_t>(seq)) b->count += (lens[i] - 1) / seq;  // batch.rs:63-67
    b->ends.push_back(b->count);
    at += lens[i];
  }
  b->seed = seed;
  if (b->count < b->batch) {
    delete b;
    return nullptr;
  }
  b->permute();
  return b;
}
void* or_batcher_new(const uint32_t* tokens, size_t n, int seq, int batch, uint64_t seed) {
  return or_batcher_new_shards(tokens, &n, 1, seq, batch, seed);
}
void or_batcher_free(void* b) { delete static_cast<Batcher*>(b); }
size_t or_batcher_num_sequences(void* b) { return static_cast<Batcher*>(b)->count; }
// batch.rs:213-240
void or_batcher_next(void* bp, int32_t* inputs, int32_t* targets, uint64_t* epoch, uint64_t* index) {
  Batcher* b = static_cast<Batcher*>(bp);
  if (b->next == b->count / b->batch) {
    b->epoch += 1;
    b->next = 0;
    b->permute();
  }
  for (size_t r = 0; r < b->batch; ++r) {
    const uint32_t* w = b->window(b->order[b->next * b->batch + r]);
    for (size_t t = 0; t < b->seq; ++t) {
      inputs[r * b->seq + t] = static_cast<int32_t>(w[t]);
      targets[r * b->seq + t] = static_cast<int32_t>(w[t + 1]);
    }
  }
  *epoch = b->epoch;
  *index = b->next;
  b->next += 1;
}

}  // extern "C"
