// The midman C ABI (include/midman_api.h): the reference's lab API
// (crates/midman-api/src/ffi.rs, lab.rs) backed by the GPU trainer, plus the
// training entry points. State is thread-local; every call but the accessors
// clears the text, floats and error buffers first (ffi.rs:119-145).
#include <cuda_runtime.h>
#include "nccl_api.h"

#include <cmath>
#include <cstdlib>
#include <cstring>
#include <exception>
#include <memory>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include "../../include/midman_api.h"
#include "host.h"
#include "json.h"
#include "shard.h"
#include "state.h"
#include "trainer.h"

namespace {

using namespace mm;

// Error kinds, mapped to the reference's status codes (ffi.rs:101-109).
struct ArgumentError : std::runtime_error { using std::runtime_error::runtime_error; };
struct ConfigError : std::runtime_error { using std::runtime_error::runtime_error; };
struct IndexError : std::runtime_error { using std::runtime_error::runtime_error; };
struct DeviceError : std::runtime_error { using std::runtime_error::runtime_error; };

constexpr uint64_t kMaxParams = 8000000;  // lab.rs:22
constexpr uint64_t kMaxTokens = 4096;     // lab.rs:25
const char* kConfigFields[MIDMAN_CONFIG_LEN] = {"vocab_size", "d_model", "n_layers", "n_heads", "n_kv_heads",
                                                "d_ff", "max_seq_len", "rope_theta", "norm_eps", "tie_embeddings"};
const char* kHyperFields[MIDMAN_HYPER_LEN] = {"max_lr", "min_lr", "warmup_steps", "total_steps",
                                              "weight_decay", "clip_norm", "beta1", "beta2"};

struct Hyper {
  float max_lr, min_lr;
  uint64_t warmup, total;
  float weight_decay, clip_norm, beta1, beta2;
};

// lab.rs:142-153 + the step state of Lab
struct Lab {
  ModelConfig cfg;
  Hyper hyper;
  int batch = 0, seq = 0;
  std::unique_ptr<Trainer> trainer;
  std::vector<int32_t> inputs, targets;
  uint64_t step = 0;
  bool has_loss = false;
  float last_loss = 0.0f;
  std::vector<float> last_norms;
};

struct Train {
  Hyper hyper;
  std::unique_ptr<Trainer> trainer;
  uint64_t step = 0;
};

struct State {
  std::vector<std::unique_ptr<Lab>> labs;
  std::vector<std::unique_ptr<Train>> trains;
  std::vector<std::unique_ptr<Batcher>> batchers;
  std::vector<uint8_t> text;
  std::vector<float> floats;
  std::vector<uint8_t> error;
};

thread_local State g;

void set_text(const std::string& s) { g.text.assign(s.begin(), s.end()); }
void set_error(const std::string& s) { g.error.assign(s.begin(), s.end()); }

template <class F>
int32_t run(F&& body) {
  g.text.clear();
  g.floats.clear();
  g.error.clear();
  try {
    return body();
  } catch (const ArgumentError& e) {
    set_error(e.what());
    return MIDMAN_ERR_ARGUMENT;
  } catch (const std::invalid_argument& e) {
    set_error(e.what());
    return MIDMAN_ERR_ARGUMENT;
  } catch (const ConfigError& e) {
    set_error(e.what());
    return MIDMAN_ERR_CONFIG;
  } catch (const IndexError& e) {
    set_error(e.what());
    return MIDMAN_ERR_INDEX;
  } catch (const std::out_of_range& e) {
    set_error(e.what());
    return MIDMAN_ERR_INDEX;
  } catch (const DeviceError& e) {
    set_error(e.what());
    return MIDMAN_ERR_DEVICE;
  } catch (const ShardError& e) {
    set_error(e.what());
    return MIDMAN_ERR_OTHER;
  } catch (const StateShapeError& e) {
    set_error(e.what());
    return MIDMAN_ERR_SHAPE;
  } catch (const std::bad_alloc&) {
    set_error("internal error: out of host memory");
    return MIDMAN_ERR_PANIC;
  } catch (const std::exception& e) {
    set_error(e.what());
    return MIDMAN_ERR_OTHER;
  } catch (...) {
    set_error("internal error: an exception with no message");
    return MIDMAN_ERR_PANIC;
  }
}

const double* read_f64s(const double* p, const char* what) {
  if (!p) throw ArgumentError(std::string(what) + " is a null pointer");
  if (reinterpret_cast<uintptr_t>(p) & 7u) throw ArgumentError(std::string(what) + " is not aligned for f64");
  return p;
}

std::string fmt(double v) {
  JsonWriter w;
  w.number(v);
  return w.finish();
}

// ffi.rs:165-181
uint64_t as_count(double v, const char* name) {
  if (std::isfinite(v) && v >= 0.0 && std::floor(v) == v && v <= 4294967295.0) return static_cast<uint64_t>(v);
  throw ArgumentError(std::string(name) + " must be a whole number from 0 to 4294967295, got " + fmt(v));
}
float as_finite_f32(double v, const char* name) {
  if (std::isfinite(v) && std::fabs(v) <= 3.4028234663852886e38) return static_cast<float>(v);
  throw ArgumentError(std::string(name) + " must be a finite number that fits in f32, got " + fmt(v));
}

ModelConfig config_from(const double* v) {
  ModelConfig c;
  c.vocab = as_count(v[0], kConfigFields[0]);
  c.d_model = as_count(v[1], kConfigFields[1]);
  c.n_layers = as_count(v[2], kConfigFields[2]);
  c.n_heads = as_count(v[3], kConfigFields[3]);
  c.n_kv_heads = as_count(v[4], kConfigFields[4]);
  c.d_ff = as_count(v[5], kConfigFields[5]);
  c.max_seq_len = as_count(v[6], kConfigFields[6]);
  c.rope_theta = as_finite_f32(v[7], kConfigFields[7]);
  c.norm_eps = as_finite_f32(v[8], kConfigFields[8]);
  c.tie = v[9] != 0.0;
  return c;
}

std::vector<double> config_values(const ModelConfig& c) {
  return {static_cast<double>(c.vocab),       static_cast<double>(c.d_model),  static_cast<double>(c.n_layers),
          static_cast<double>(c.n_heads),     static_cast<double>(c.n_kv_heads), static_cast<double>(c.d_ff),
          static_cast<double>(c.max_seq_len), static_cast<double>(c.rope_theta), static_cast<double>(c.norm_eps),
          c.tie ? 1.0 : 0.0};
}

Hyper hyper_from(const double* v) {
  Hyper h;
  h.max_lr = as_finite_f32(v[0], kHyperFields[0]);
  h.min_lr = as_finite_f32(v[1], kHyperFields[1]);
  h.warmup = as_count(v[2], kHyperFields[2]);
  h.total = as_count(v[3], kHyperFields[3]);
  h.weight_decay = as_finite_f32(v[4], kHyperFields[4]);
  h.clip_norm = as_finite_f32(v[5], kHyperFields[5]);
  h.beta1 = as_finite_f32(v[6], kHyperFields[6]);
  h.beta2 = as_finite_f32(v[7], kHyperFields[7]);
  return h;
}

// WarmupCosine::new (schedule.rs:23-46) and AdamW::new (adamw.rs:47-64) checks.
void validate_hyper(const Hyper& h) {
  if (!(std::isfinite(h.clip_norm) && h.clip_norm > 0.0f))
    throw ArgumentError("clip_norm must be positive and finite, got " + fmt(h.clip_norm));
  if (!(std::isfinite(h.max_lr) && h.max_lr > 0.0f))
    throw ArgumentError("schedule: max_lr must be positive and finite, got " + fmt(h.max_lr));
  if (!(std::isfinite(h.min_lr) && h.min_lr >= 0.0f && h.min_lr <= h.max_lr))
    throw ArgumentError("schedule: min_lr must be in [0, max_lr = " + fmt(h.max_lr) + "], got " + fmt(h.min_lr));
  if (h.warmup >= h.total)
    throw ArgumentError("schedule: warmup_steps " + std::to_string(h.warmup) + " must be below total_steps " +
                        std::to_string(h.total));
  if (!(h.beta1 >= 0.0f && h.beta1 < 1.0f)) throw ArgumentError("adamw: beta1 must be in [0, 1), got " + fmt(h.beta1));
  if (!(h.beta2 >= 0.0f && h.beta2 < 1.0f)) throw ArgumentError("adamw: beta2 must be in [0, 1), got " + fmt(h.beta2));
  if (!(std::isfinite(h.weight_decay) && h.weight_decay >= 0.0f))
    throw ArgumentError("adamw: weight_decay must be finite and not negative, got " + fmt(h.weight_decay));
}

uint64_t validated_param_count(const ModelConfig& c) {
  ParamBreakdown b;
  std::string err;
  if (!param_breakdown(c, &b, &err)) throw ConfigError("invalid config: " + err);
  return b.total();
}

AdamHyper adam_of(const Hyper& h) {
  AdamHyper a;
  a.beta1 = h.beta1;
  a.beta2 = h.beta2;
  a.eps = 1e-8f;  // lab.rs:192
  a.weight_decay = h.weight_decay;
  a.clip_norm = h.clip_norm;
  return a;
}

Lab& lab_ref(uint32_t handle) {
  if (handle == 0 || handle > g.labs.size() || !g.labs[handle - 1])
    throw ArgumentError(std::to_string(handle) + " is not a live lab handle");
  return *g.labs[handle - 1];
}

Train& train_ref(uint32_t handle) {
  if (handle == 0 || handle > g.trains.size() || !g.trains[handle - 1])
    throw ArgumentError(std::to_string(handle) + " is not a live trainer handle");
  return *g.trains[handle - 1];
}

template <class T>
uint32_t insert(std::vector<std::unique_ptr<T>>& v, std::unique_ptr<T> item) {
  for (size_t i = 0; i < v.size(); ++i)
    if (!v[i]) {
      v[i] = std::move(item);
      return static_cast<uint32_t>(i + 1);
    }
  v.push_back(std::move(item));
  return static_cast<uint32_t>(v.size());
}

int host_threads() {
  const char* e = std::getenv("MIDMAN_INIT_THREADS");
  int n = e ? std::atoi(e) : 0;
  if (n <= 0) {
    n = static_cast<int>(std::thread::hardware_concurrency());
    if (n <= 0) n = 1;
    if (n > 32) n = 32;
  }
  return n;
}

}  // namespace

extern "C" {

uint32_t midman_abi_version(void) { return MIDMAN_ABI_VERSION; }

uint8_t* midman_alloc(uint32_t len) {
  void* p = nullptr;
  if (posix_memalign(&p, 8, len ? len : 1) != 0) return nullptr;
  return static_cast<uint8_t*>(p);
}

void midman_free(uint8_t* ptr, uint32_t) { std::free(ptr); }

const uint8_t* midman_text_ptr(void) { return g.text.data(); }
uint32_t midman_text_len(void) { return static_cast<uint32_t>(g.text.size()); }
const float* midman_floats_ptr(void) { return g.floats.data(); }
uint32_t midman_floats_len(void) { return static_cast<uint32_t>(g.floats.size()); }
const uint8_t* midman_error_ptr(void) { return g.error.data(); }
uint32_t midman_error_len(void) { return static_cast<uint32_t>(g.error.size()); }

// ffi.rs:333-370
int32_t midman_describe(void) {
  return run([] {
    JsonWriter w;
    w.begin_object();
    w.key("abi").integer(MIDMAN_ABI_VERSION);
    w.key("version").string("0.0.1");
    w.key("config_fields").begin_array();
    for (auto f : kConfigFields) w.string(f);
    w.end_array();
    w.key("hyper_fields").begin_array();
    for (auto f : kHyperFields) w.string(f);
    w.end_array();
    w.key("limits").begin_object();
    w.key("max_params").integer(kMaxParams);
    w.key("max_tokens").integer(kMaxTokens);
    w.end_object();
    w.key("presets").begin_array();
    for (int i = 0; i < kNumPresets; ++i) {
      const ModelConfig c = preset_config(i);
      w.begin_object();
      w.key("name").string(preset_name(i));
      w.key("config").begin_array();
      for (double v : config_values(c)) w.number(v);
      w.end_array();
      w.key("params").integer(validated_param_count(c));
      w.end_object();
    }
    w.end_array();
    w.end_object();
    set_text(w.finish());
    return MIDMAN_OK;
  });
}

// ffi.rs:378-395
int32_t midman_preset_config(uint32_t index, double* out) {
  return run([&] {
    if (index >= kNumPresets) throw ArgumentError("there is no preset " + std::to_string(index));
    if (!out || (reinterpret_cast<uintptr_t>(out) & 7u)) throw ArgumentError("out is null or not aligned for f64");
    const auto v = config_values(preset_config(static_cast<int>(index)));
    std::memcpy(out, v.data(), MIDMAN_CONFIG_LEN * sizeof(double));
    return MIDMAN_OK;
  });
}

// ffi.rs:403-434
int32_t midman_config_report(const double* config) {
  return run([&] {
    const ModelConfig c = config_from(read_f64s(config, "config"));
    JsonWriter w;
    w.begin_object();
    ParamBreakdown b;
    std::string err;
    if (param_breakdown(c, &b, &err)) {
      w.key("valid").boolean(true);
      w.key("head_dim").integer(c.head_dim());
      w.key("kv_dim").integer(c.kv_dim());
      w.key("params").begin_object();
      w.key("embedding").integer(b.embedding);
      w.key("attention").integer(b.attention);
      w.key("mlp").integer(b.mlp);
      w.key("norms").integer(b.norms);
      w.key("lm_head").integer(b.lm_head);
      w.key("total").integer(b.total());
      w.end_object();
    } else {
      w.key("valid").boolean(false);
      w.key("error").string("invalid config: " + err);
    }
    w.end_object();
    set_text(w.finish());
    return MIDMAN_OK;
  });
}

// ffi.rs:442-460, report.rs:43-50
int32_t midman_rope_table(uint32_t head_dim, uint32_t max_seq_len, double theta) {
  return run([&] {
    const float t = as_finite_f32(theta, "theta");
    if (head_dim == 0 || (head_dim & 1u))
      throw ArgumentError("rope: head_dim must be even and positive, got " + std::to_string(head_dim));
    if (max_seq_len == 0) throw ArgumentError("rope: max_seq_len must be at least 1");
    if (!(std::isfinite(t) && t > 0.0f)) throw ArgumentError("rope: theta must be positive and finite, got " + fmt(t));
    std::vector<float> c, s;
    rope_tables(head_dim, max_seq_len, t, c, s);
    g.floats = c;
    g.floats.insert(g.floats.end(), s.begin(), s.end());
    JsonWriter w;
    w.begin_object();
    w.key("positions").integer(max_seq_len);
    w.key("half").integer(head_dim / 2);
    w.end_object();
    set_text(w.finish());
    return MIDMAN_OK;
  });
}

// ffi.rs:473-508 and Lab::new (lab.rs:159-216)
uint32_t midman_lab_create(const double* config, const double* hyper, uint32_t seed_lo, uint32_t seed_hi,
                           uint32_t batch, uint32_t seq) {
  const int32_t status = run([&]() -> int32_t {
    const ModelConfig cfg = config_from(read_f64s(config, "config"));
    const Hyper h = hyper_from(read_f64s(hyper, "hyper"));
    const uint64_t params = validated_param_count(cfg);
    if (params > kMaxParams)
      throw ArgumentError("the lab builds models up to " + std::to_string(kMaxParams) + " parameters, this one has " +
                          std::to_string(params));
    if (batch == 0 || seq == 0) throw ArgumentError("the lab needs at least one sequence of at least one token");
    if (seq > cfg.max_seq_len)
      throw ArgumentError("sequence length " + std::to_string(seq) + " exceeds the model's max_seq_len " +
                          std::to_string(cfg.max_seq_len));
    if (static_cast<uint64_t>(batch) * seq > kMaxTokens)
      throw ArgumentError("the lab task is limited to " + std::to_string(kMaxTokens) + " tokens, got " +
                          std::to_string(batch) + " x " + std::to_string(seq));
    validate_hyper(h);
    auto lab = std::make_unique<Lab>();
    lab->cfg = cfg;
    lab->hyper = h;
    lab->batch = static_cast<int>(batch);
    lab->seq = static_cast<int>(seq);
    lab->trainer = std::make_unique<Trainer>(cfg, lab->batch, lab->seq, kPrecision3xTF32);
    HostRng rng((static_cast<uint64_t>(seed_hi) << 32) | seed_lo);
    lab->trainer->init_params(rng, 0.02f, host_threads());
    // the task: batch sequences of seq + 1 ids from the same generator (lab.rs:196-204)
    for (uint32_t b = 0; b < batch; ++b) {
      std::vector<int32_t> toks(seq + 1);
      for (auto& t : toks) t = static_cast<int32_t>(rng.below(cfg.vocab));
      lab->inputs.insert(lab->inputs.end(), toks.begin(), toks.end() - 1);
      lab->targets.insert(lab->targets.end(), toks.begin() + 1, toks.end());
    }
    return static_cast<int32_t>(insert(g.labs, std::move(lab)));
  });
  return status > 0 ? static_cast<uint32_t>(status) : 0u;
}

// ffi.rs:518-532, Lab::step (lab.rs:251-289)
int32_t midman_lab_step(uint32_t handle, uint32_t steps) {
  return run([&] {
    Lab& lab = lab_ref(handle);
    for (uint32_t i = 0; i < steps; ++i) {
      const float lr = schedule_lr(lab.hyper.max_lr, lab.hyper.min_lr, lab.hyper.warmup, lab.hyper.total, lab.step);
      const StepOut r = lab.trainer->train_step(lab.inputs.data(), lab.targets.data(), lr, adam_of(lab.hyper));
      if (!r.ok) {
        if (!std::isfinite(r.loss))
          set_error("the loss is " + std::string(std::isnan(r.loss) ? "NaN" : (r.loss > 0 ? "inf" : "-inf")) +
                    ", not a finite number");
        else
          set_error("clip: the gradient norm is not finite");
        return MIDMAN_STOPPED;
      }
      lab.last_norms = lab.trainer->grad_norms();
      lab.step += 1;
      lab.has_loss = true;
      lab.last_loss = r.loss;
      g.floats.push_back(r.loss);
      g.floats.push_back(r.grad_norm);
      g.floats.push_back(lr);
    }
    return MIDMAN_OK;
  });
}

// ffi.rs:539-570, Lab::eval (lab.rs:291-308)
int32_t midman_lab_eval(uint32_t handle) {
  return run([&] {
    Lab& lab = lab_ref(handle);
    std::vector<int32_t> pred(lab.inputs.size());
    const float loss = lab.trainer->eval(lab.inputs.data(), lab.targets.data(), lab.batch, lab.seq, pred.data());
    size_t correct = 0;
    for (size_t i = 0; i < pred.size(); ++i) correct += pred[i] == lab.targets[i];
    JsonWriter w;
    w.begin_object();
    w.key("step").integer(lab.step);
    w.key("loss").number(loss);
    w.key("accuracy").number(static_cast<float>(correct) / static_cast<float>(pred.size()));
    w.key("batch").integer(lab.batch);
    w.key("seq").integer(lab.seq);
    const std::vector<int32_t>* arrays[3] = {&lab.inputs, &lab.targets, &pred};
    const char* names[3] = {"inputs", "targets", "predictions"};
    for (int a = 0; a < 3; ++a) {
      w.key(names[a]).begin_array();
      for (int b = 0; b < lab.batch; ++b) {
        w.begin_array();
        for (int t = 0; t < lab.seq; ++t) w.integer(static_cast<uint64_t>((*arrays[a])[b * lab.seq + t]));
        w.end_array();
      }
      w.end_array();
    }
    w.end_object();
    set_text(w.finish());
    return MIDMAN_OK;
  });
}

// ffi.rs:576-602, Lab::param_stats (lab.rs:329-343)
int32_t midman_lab_stats(uint32_t handle) {
  return run([&] {
    Lab& lab = lab_ref(handle);
    const ParamLayout& L = lab.trainer->layout();
    std::vector<float> params(L.total);
    lab.trainer->read_params(params.data());
    JsonWriter w;
    w.begin_object();
    w.key("step").integer(lab.step);
    w.key("last_loss").optional_number(lab.has_loss, lab.last_loss);
    w.key("num_parameters").integer(L.total);
    w.key("params").begin_array();
    for (size_t i = 0; i < L.tensors.size(); ++i) {
      const TensorInfo& t = L.tensors[i];
      double ss = 0.0;
      for (uint64_t k = 0; k < t.numel; ++k) ss += static_cast<double>(params[t.offset + k]) * params[t.offset + k];
      const float rms = t.numel ? static_cast<float>(std::sqrt(ss / static_cast<double>(t.numel))) : 0.0f;
      w.begin_object();
      w.key("name").string(t.name);
      w.key("shape").begin_array();
      for (auto d : t.shape) w.integer(d);
      w.end_array();
      w.key("rms").number(rms);
      w.key("grad_norm").optional_number(i < lab.last_norms.size(), i < lab.last_norms.size() ? lab.last_norms[i] : 0);
      w.end_object();
    }
    w.end_array();
    w.end_object();
    set_text(w.finish());
    return MIDMAN_OK;
  });
}

// ffi.rs:608-620, Lab::attention (lab.rs:310-327)
int32_t midman_lab_attention(uint32_t handle, uint32_t sequence) {
  return run([&] {
    Lab& lab = lab_ref(handle);
    if (sequence >= static_cast<uint32_t>(lab.batch))
      throw ArgumentError("sequence " + std::to_string(sequence) + " does not exist, the task has " +
                          std::to_string(lab.batch));
    const size_t n = lab.cfg.n_layers * lab.cfg.n_heads * static_cast<size_t>(lab.seq) * lab.seq;
    g.floats.resize(n);
    lab.trainer->attention_maps(lab.inputs.data() + static_cast<size_t>(sequence) * lab.seq, 1, lab.seq,
                                g.floats.data());
    JsonWriter w;
    w.begin_object();
    w.key("layers").integer(lab.cfg.n_layers);
    w.key("heads").integer(lab.cfg.n_heads);
    w.key("seq").integer(lab.seq);
    w.end_object();
    set_text(w.finish());
    return MIDMAN_OK;
  });
}

// ffi.rs:626-638, Lab::embedding (lab.rs:318-327)
int32_t midman_lab_embedding(uint32_t handle) {
  return run([&] {
    Lab& lab = lab_ref(handle);
    const uint64_t n = lab.cfg.vocab * lab.cfg.d_model;
    g.floats.resize(n);
    lab.trainer->read_tensor(lab.trainer->layout().embed, n, g.floats.data(), 0);
    JsonWriter w;
    w.begin_object();
    w.key("rows").integer(lab.cfg.vocab);
    w.key("cols").integer(lab.cfg.d_model);
    w.end_object();
    set_text(w.finish());
    return MIDMAN_OK;
  });
}

// ffi.rs:641-647
int32_t midman_lab_destroy(uint32_t handle) {
  return run([&] {
    lab_ref(handle);
    g.labs[handle - 1].reset();
    return MIDMAN_OK;
  });
}

// ---------------------------------------------------------------- training

int32_t midman_nccl_unique_id(uint8_t* out128) {
  return run([&] {
    if (!out128) throw ArgumentError("out is a null pointer");
    ncclUniqueId id;
    const ncclResult_t r = nccl().GetUniqueId(&id);
    if (r != ncclSuccess) throw DeviceError(std::string("ncclGetUniqueId: ") + nccl().GetErrorString(r));
    static_assert(sizeof(id) == 128, "NCCL unique id is 128 bytes");
    std::memcpy(out128, &id, sizeof(id));
    return MIDMAN_OK;
  });
}

uint32_t midman_train_create(const double* config, const double* hyper, uint32_t seed_lo, uint32_t seed_hi,
                             uint32_t batch, uint32_t seq, uint32_t precision, uint32_t world, uint32_t rank,
                             const uint8_t* nccl_id) {
  const int32_t status = run([&]() -> int32_t {
    const ModelConfig cfg = config_from(read_f64s(config, "config"));
    const Hyper h = hyper_from(read_f64s(hyper, "hyper"));
    validated_param_count(cfg);
    validate_hyper(h);
    if (batch == 0 || seq == 0) throw ArgumentError("batch and seq must be at least 1");
    auto t = std::make_unique<Train>();
    t->hyper = h;
    try {
      t->trainer = std::make_unique<Trainer>(cfg, static_cast<int>(batch), static_cast<int>(seq),
                                             static_cast<int>(precision), static_cast<int>(world),
                                             static_cast<int>(rank), nccl_id);
    } catch (const std::runtime_error& e) {
      if (dynamic_cast<const std::invalid_argument*>(&e)) throw;
      throw DeviceError(e.what());
    }
    HostRng rng((static_cast<uint64_t>(seed_hi) << 32) | seed_lo);
    t->trainer->init_params(rng, 0.02f, host_threads());
    return static_cast<int32_t>(insert(g.trains, std::move(t)));
  });
  return status > 0 ? static_cast<uint32_t>(status) : 0u;
}

namespace {
int32_t record_step(Train& t, const StepOut& r, float lr) {
  g.floats.push_back(r.loss);
  g.floats.push_back(r.grad_norm);
  g.floats.push_back(lr);
  if (!r.ok) {
    g.floats.resize(g.floats.size() - 3);
    set_error(std::isfinite(r.loss) ? "clip: the gradient norm is not finite"
                                    : "the loss is not a finite number");
    return MIDMAN_STOPPED;
  }
  t.step += 1;
  return MIDMAN_OK;
}
}  // namespace

int32_t midman_train_step(uint32_t handle, const int32_t* inputs, const int32_t* targets) {
  return run([&] {
    Train& t = train_ref(handle);
    if (!inputs || !targets) throw ArgumentError("inputs and targets must not be null");
    const float lr = schedule_lr(t.hyper.max_lr, t.hyper.min_lr, t.hyper.warmup, t.hyper.total, t.step);
    return record_step(t, t.trainer->train_step(inputs, targets, lr, adam_of(t.hyper)), lr);
  });
}

int32_t midman_train_stage(uint32_t handle, const int32_t* inputs, const int32_t* targets) {
  return run([&] {
    Train& t = train_ref(handle);
    if (!inputs || !targets) throw ArgumentError("inputs and targets must not be null");
    t.trainer->stage_batch(inputs, targets);
    return MIDMAN_OK;
  });
}

int32_t midman_train_step_staged(uint32_t handle, uint32_t steps) {
  return run([&] {
    Train& t = train_ref(handle);
    for (uint32_t i = 0; i < steps; ++i) {
      const float lr = schedule_lr(t.hyper.max_lr, t.hyper.min_lr, t.hyper.warmup, t.hyper.total, t.step);
      const int32_t rc = record_step(t, t.trainer->step_staged(lr, adam_of(t.hyper)), lr);
      if (rc != MIDMAN_OK) return rc;
    }
    return MIDMAN_OK;
  });
}

int32_t midman_train_loss_and_grads(uint32_t handle, const int32_t* inputs, const int32_t* targets) {
  return run([&] {
    Train& t = train_ref(handle);
    if (!inputs || !targets) throw ArgumentError("inputs and targets must not be null");
    g.floats.push_back(t.trainer->loss_and_grads(inputs, targets));
    return MIDMAN_OK;
  });
}

int32_t midman_train_read(uint32_t handle, uint32_t which, uint32_t index) {
  return run([&] {
    Train& t = train_ref(handle);
    if (which > 3) throw ArgumentError("which must be 0 (params), 1 (grads), 2 (m) or 3 (v)");
    const ParamLayout& L = t.trainer->layout();
    uint64_t off = 0, n = L.total;
    if (index != 0xFFFFFFFFu) {
      if (index >= L.tensors.size())
        throw IndexError("tensor index " + std::to_string(index) + " is out of range for " +
                         std::to_string(L.tensors.size()) + " tensors");
      off = L.tensors[index].offset;
      n = L.tensors[index].numel;
    }
    g.floats.resize(n);
    t.trainer->read_tensor(off, n, g.floats.data(), static_cast<int>(which));
    return MIDMAN_OK;
  });
}

int32_t midman_train_params(uint32_t handle, uint32_t index) { return midman_train_read(handle, 0, index); }

int32_t midman_train_grads(uint32_t handle, uint32_t index) { return midman_train_read(handle, 1, index); }

int32_t midman_train_load(uint32_t handle, const float* values, uint64_t len) {
  return run([&] {
    Train& t = train_ref(handle);
    if (!values) throw ArgumentError("values is a null pointer");
    if (len != t.trainer->layout().total)
      throw ArgumentError("expected " + std::to_string(t.trainer->layout().total) + " values, got " +
                          std::to_string(len));
    t.trainer->load_params(values);
    return MIDMAN_OK;
  });
}

namespace {
std::string path_from(const uint8_t* path, uint32_t len) {
  if (!path || len == 0) throw ArgumentError("the path must not be empty");
  return std::string(reinterpret_cast<const char*>(path), len);
}

// TrainConfig of this run (config.rs:16-41): the global batch, the schedule and
// AdamW settings it was created with, and the data-order seed of its batcher.
TrainSettings settings_of(const Train& t, uint32_t seed_lo, uint32_t seed_hi) {
  TrainSettings s;
  s.batch_size = static_cast<uint64_t>(t.trainer->batch()) * static_cast<uint64_t>(t.trainer->world());
  s.seq_len = static_cast<uint64_t>(t.trainer->seq());
  s.seed = (static_cast<uint64_t>(seed_hi) << 32) | seed_lo;
  s.max_lr = t.hyper.max_lr;
  s.min_lr = t.hyper.min_lr;
  s.warmup_steps = t.hyper.warmup;
  s.total_steps = t.hyper.total;
  s.beta1 = t.hyper.beta1;
  s.beta2 = t.hyper.beta2;
  s.eps = adam_of(t.hyper).eps;
  s.weight_decay = t.hyper.weight_decay;
  s.clip_norm = t.hyper.clip_norm;
  return s;
}

std::vector<StateParam> state_params(const ParamLayout& L) {
  std::vector<StateParam> out;
  for (const TensorInfo& ti : L.tensors) {
    StateParam p;
    p.name = ti.name;
    for (auto d : ti.shape) p.shape.push_back(static_cast<uint64_t>(d));
    p.offset = ti.offset;
    p.count = ti.numel;
    out.push_back(std::move(p));
  }
  return out;
}

// "sharding": {"optimizer": bool, "ranges": [[begin, end] per rank], "buckets": [[begin, end]...]}
void write_sharding(JsonWriter& w, const Trainer& tr) {
  w.key("sharding").begin_object();
  w.key("optimizer").boolean(tr.optimizer_sharded());
  w.key("world").integer(tr.world());
  w.key("rank").integer(tr.rank());
  w.key("ranges").begin_array();
  for (int r = 0; r < tr.world(); ++r) {
    w.begin_array();
    w.integer(tr.shard_begin(r));
    w.integer(tr.shard_end(r));
    w.end_array();
  }
  w.end_array();
  w.key("buckets").begin_array();
  for (const auto& b : tr.buckets()) {
    w.begin_array();
    w.integer(b.first);
    w.integer(b.second);
    w.end_array();
  }
  w.end_array();
  w.end_object();
}

void write_progress(JsonWriter& w, const Progress& p) {
  w.begin_object();
  w.key("step").integer(p.step);
  w.key("epoch").integer(p.epoch);
  w.key("position").integer(p.position);
  w.end_object();
}
}  // namespace

int32_t midman_train_save(uint32_t handle, const uint8_t* path, uint32_t path_len, uint32_t data_seed_lo,
                          uint32_t data_seed_hi, uint64_t epoch, uint64_t position) {
  return run([&] {
    Train& t = train_ref(handle);
    const std::string file = path_from(path, path_len);
    Progress p;
    p.step = t.step;
    p.epoch = epoch;
    p.position = position;
    Trainer& tr = *t.trainer;
    if (tr.optimizer_sharded() && tr.world() > 1) {
      // collective: every rank gathers the moments from their owners; rank 0 writes
      const uint64_t total = tr.layout().total;
      std::vector<float> m(total), v(total);
      tr.read_tensor(0, total, m.data(), 2);
      tr.read_tensor(0, total, v.data(), 3);
      if (tr.rank() != 0) return MIDMAN_OK;
      save_state(file, state_params(tr.layout()), p, settings_of(t, data_seed_lo, data_seed_hi),
                 [&](int which, uint64_t offset, uint64_t n, float* out) {
                   if (which == 2 || which == 3)
                     std::memcpy(out, (which == 2 ? m : v).data() + offset, n * 4);
                   else
                     tr.read_tensor(offset, n, out, which);
                 });
      return MIDMAN_OK;
    }
    save_state(file, state_params(tr.layout()), p, settings_of(t, data_seed_lo, data_seed_hi),
               [&](int which, uint64_t offset, uint64_t n, float* out) { tr.read_tensor(offset, n, out, which); });
    return MIDMAN_OK;
  });
}

int32_t midman_shard_plan(const double* config, uint32_t world) {
  return run([&] {
    const ModelConfig c = config_from(read_f64s(config, "config"));
    const std::string bad = validate_config(c);
    if (!bad.empty()) throw ConfigError(bad);
    if (world < 1 || world > 4096) throw ArgumentError("world must be between 1 and 4096");
    const ParamLayout L = param_layout(c);
    const uint64_t block = static_cast<uint64_t>(norm_block_elems(static_cast<long long>(L.total)));
    const std::vector<uint64_t> bounds = shard_bounds(L.total, static_cast<int>(world), block, kNormBlocks);
    JsonWriter w;
    w.begin_object();
    w.key("params").integer(L.total);
    w.key("norm_block").integer(block);
    w.key("norm_blocks").integer(kNormBlocks);
    w.key("ranges").begin_array();
    for (uint32_t r = 0; r < world; ++r) {
      w.begin_array();
      w.integer(bounds[r]);
      w.integer(bounds[r + 1]);
      w.end_array();
    }
    w.end_array();
    w.key("buckets").begin_array();
    for (const auto& b : gradient_buckets(c, L)) {
      w.begin_array();
      w.integer(b.first);
      w.integer(b.second);
      w.end_array();
    }
    w.end_array();
    w.end_object();
    set_text(w.finish());
    return MIDMAN_OK;
  });
}

int32_t midman_train_shard_optimizer(uint32_t handle, uint32_t enable) {
  return run([&] {
    Train& t = train_ref(handle);
    t.trainer->shard_optimizer(enable != 0);
    JsonWriter w;
    w.begin_object();
    write_sharding(w, *t.trainer);
    w.end_object();
    set_text(w.finish());
    return MIDMAN_OK;
  });
}

int32_t midman_train_restore(uint32_t handle, const uint8_t* path, uint32_t path_len, uint32_t data_seed_lo,
                             uint32_t data_seed_hi) {
  return run([&] {
    Train& t = train_ref(handle);
    const std::string file = path_from(path, path_len);
    const ParamLayout& L = t.trainer->layout();
    LoadedState st = load_state(file, state_params(L), L.total, settings_of(t, data_seed_lo, data_seed_hi));
    t.trainer->restore(st.params.data(), st.m.empty() ? nullptr : st.m.data(), st.v.empty() ? nullptr : st.v.data(),
                       st.progress.step);
    t.step = st.progress.step;
    JsonWriter w;
    write_progress(w, st.progress);
    set_text(w.finish());
    return MIDMAN_OK;
  });
}

int32_t midman_state_inspect(const uint8_t* path, uint32_t path_len) {
  return run([&] {
    const SafeFile f = load_safetensors(path_from(path, path_len));
    JsonWriter w;
    w.begin_object();
    w.key("metadata").begin_object();
    for (const auto& [k, v] : f.metadata) w.key(k).string(v);
    w.end_object();
    w.key("tensors").begin_array();
    for (const SafeTensor& t : f.tensors) {
      w.begin_object();
      w.key("name").string(t.name);
      w.key("shape").begin_array();
      for (auto d : t.shape) w.integer(d);
      w.end_array();
      w.key("data_offsets").begin_array().integer(t.begin).integer(t.end).end_array();
      w.end_object();
    }
    w.end_array();
    const auto fmt = f.metadata.find("format");
    if (fmt != f.metadata.end() && fmt->second == "midman-training-state") {  // its header entries must hold
      w.key("progress");
      write_progress(w, progress_of(f.metadata));
    }
    w.end_object();
    set_text(w.finish());
    return MIDMAN_OK;
  });
}

int32_t midman_train_describe(uint32_t handle) {
  return run([&] {
    Train& t = train_ref(handle);
    const ParamLayout& L = t.trainer->layout();
    JsonWriter w;
    w.begin_object();
    w.key("params").integer(L.total);
    w.key("steps").integer(t.step);
    w.key("kernel_launches").integer(t.trainer->kernel_launches());
    write_sharding(w, *t.trainer);
    w.key("profile").begin_object();
    for (const auto& e : t.trainer->profile()) {
      w.key(e.first).begin_object();
      w.key("launches").integer(e.second.launches);
      w.key("ms").number(e.second.ms);
      w.key("flops").number(e.second.flops);
      w.end_object();
    }
    w.end_object();
    w.key("profile_gemm").begin_object();
    for (const auto& e : t.trainer->gemm_profile()) {
      w.key(e.first).begin_object();
      w.key("launches").integer(e.second.launches);
      w.key("ms").number(e.second.ms);
      w.key("flops").number(e.second.flops);
      w.end_object();
    }
    w.end_object();
    w.key("tensors").begin_array();
    for (const TensorInfo& ti : L.tensors) {
      w.begin_object();
      w.key("name").string(ti.name);
      w.key("shape").begin_array();
      for (auto d : ti.shape) w.integer(d);
      w.end_array();
      w.key("offset").integer(ti.offset);
      w.end_object();
    }
    w.end_array();
    w.end_object();
    set_text(w.finish());
    return MIDMAN_OK;
  });
}

int32_t midman_train_eval(uint32_t handle, const int32_t* inputs, const int32_t* targets, uint32_t batch,
                          uint32_t seq) {
  return run([&] {
    Train& t = train_ref(handle);
    if (!inputs || !targets) throw ArgumentError("inputs and targets must not be null");
    if (batch == 0 || seq == 0) throw ArgumentError("batch and seq must be at least 1");
    g.floats.push_back(t.trainer->eval(inputs, targets, static_cast<int>(batch), static_cast<int>(seq), nullptr));
    return MIDMAN_OK;
  });
}

int32_t midman_train_stream(uint32_t handle, uint64_t* out) {
  return run([&] {
    Train& t = train_ref(handle);
    if (!out) throw ArgumentError("out is a null pointer");
    *out = reinterpret_cast<uint64_t>(t.trainer->stream());
    return MIDMAN_OK;
  });
}

int32_t midman_train_profile(uint32_t handle, uint32_t enable) {
  return run([&] {
    train_ref(handle).trainer->set_profile(enable != 0);
    return MIDMAN_OK;
  });
}

int32_t midman_batcher_create(const uint32_t* tokens, uint64_t n, uint32_t vocab, uint32_t seq, uint32_t batch,
                              uint32_t seed_lo, uint32_t seed_hi) {
  return run([&]() -> int32_t {
    if (!tokens && n) throw ArgumentError("tokens is a null pointer");
    auto b = std::make_unique<Batcher>(std::vector<uint32_t>(tokens, tokens + n), vocab, static_cast<int>(seq),
                                       static_cast<int>(batch), (static_cast<uint64_t>(seed_hi) << 32) | seed_lo);
    return static_cast<int32_t>(insert(g.batchers, std::move(b)));
  });
}

int32_t midman_batcher_synthetic(uint32_t token_seed, uint32_t vocab, uint64_t n, uint32_t seq, uint32_t batch,
                                 uint32_t seed_lo, uint32_t seed_hi) {
  return run([&]() -> int32_t {
    if (vocab == 0) throw ArgumentError("vocab must be at least 1");
    auto b = std::make_unique<Batcher>(synthetic_tokens(token_seed, vocab, n), vocab, static_cast<int>(seq),
                                       static_cast<int>(batch), (static_cast<uint64_t>(seed_hi) << 32) | seed_lo);
    return static_cast<int32_t>(insert(g.batchers, std::move(b)));
  });
}

int32_t midman_batcher_next(uint32_t handle, int32_t* inputs, int32_t* targets) {
  return run([&] {
    if (handle == 0 || handle > g.batchers.size() || !g.batchers[handle - 1])
      throw ArgumentError(std::to_string(handle) + " is not a live batcher handle");
    if (!inputs || !targets) throw ArgumentError("inputs and targets must not be null");
    const auto at = g.batchers[handle - 1]->next(inputs, targets);
    JsonWriter w;
    w.begin_object();
    w.key("epoch").integer(at.first);
    w.key("index").integer(at.second);
    w.key("sequences").integer(g.batchers[handle - 1]->sequences());
    w.end_object();
    set_text(w.finish());
    return MIDMAN_OK;
  });
}

namespace {
Batcher& batcher_ref(uint32_t handle) {
  if (handle == 0 || handle > g.batchers.size() || !g.batchers[handle - 1])
    throw ArgumentError(std::to_string(handle) + " is not a live batcher handle");
  return *g.batchers[handle - 1];
}

void write_place(JsonWriter& w, const Batcher& b) {
  w.key("epoch").integer(b.epoch());
  w.key("position").integer(b.position());
  w.key("sequences").integer(b.sequences());
}
}  // namespace

// TokenShard::load (shard.rs:255-262) and the header fields; the first `capacity` ids into `tokens`.
static int32_t shard_read(const uint8_t* path, uint32_t path_len, uint32_t* tokens, uint64_t capacity) {
  return run([&] {
    if (!tokens && capacity) throw ArgumentError("tokens must not be null");
    const TokenShard sh = load_token_shard(path_from(path, path_len));
    const uint64_t n = std::min<uint64_t>(capacity, sh.tokens.size());
    if (n) std::memcpy(tokens, sh.tokens.data(), n * 4);
    JsonWriter w;
    w.begin_object();
    w.key("vocab_size").integer(sh.vocab_size);
    w.key("eos").integer(sh.eos);
    w.key("tokens").integer(sh.tokens.size());
    w.key("token_width").integer(sh.vocab_size <= 65536 ? 2 : 4);
    w.end_object();
    set_text(w.finish());
    return MIDMAN_OK;
  });
}

int32_t midman_sha256(const uint8_t* data, uint64_t n, uint8_t* digest) {
  return run([&] {
    if ((!data && n) || !digest) throw ArgumentError("data and digest must not be null");
    const std::array<uint8_t, 32> d = sha256(data, n);
    std::memcpy(digest, d.data(), d.size());
    return MIDMAN_OK;
  });
}

int32_t midman_shard_write(const uint8_t* path, uint32_t path_len, uint32_t vocab_size, uint32_t eos,
                           const uint32_t* tokens, uint64_t n) {
  return run([&] {
    if (!tokens && n) throw ArgumentError("tokens must not be null");
    save_token_shard(path_from(path, path_len), vocab_size, eos, tokens, n);
    return MIDMAN_OK;
  });
}

int32_t midman_shard_read(const uint8_t* path, uint32_t path_len, uint32_t* tokens, uint64_t capacity) {
  return shard_read(path, path_len, tokens, capacity);
}

int32_t midman_shard_inspect(const uint8_t* path, uint32_t path_len) {
  return shard_read(path, path_len, nullptr, 0);
}

namespace {
struct ShardSet {
  std::vector<std::vector<uint32_t>> shards;
  uint32_t vocab = 0, eos = 0;
};

// The shard files named in `paths` ('\n'-separated), checked to share one
// vocabulary and end-of-text id (Sequences::new, batch.rs:45-58).
ShardSet load_shards(const uint8_t* paths, uint32_t paths_len) {
  const std::string all = path_from(paths, paths_len);
  ShardSet set;
  size_t start = 0;
  while (start <= all.size()) {
    size_t end = all.find('\n', start);
    if (end == std::string::npos) end = all.size();
    if (end > start) {
      TokenShard sh = load_token_shard(all.substr(start, end - start));
      if (!set.shards.empty() && (sh.vocab_size != set.vocab || sh.eos != set.eos))
        throw ArgumentError("shard " + std::to_string(set.shards.size()) + " has vocabulary size " +
                            std::to_string(sh.vocab_size) + " and end-of-text " + std::to_string(sh.eos) +
                            ", but shard 0 has " + std::to_string(set.vocab) + " and " + std::to_string(set.eos));
      set.vocab = sh.vocab_size;
      set.eos = sh.eos;
      set.shards.push_back(std::move(sh.tokens));
    }
    start = end + 1;
  }
  return set;
}
}  // namespace

int32_t midman_batcher_open(const uint8_t* paths, uint32_t paths_len, uint32_t seq, uint32_t batch,
                            uint32_t seed_lo, uint32_t seed_hi) {
  return run([&]() -> int32_t {
    ShardSet set = load_shards(paths, paths_len);
    if (set.shards.empty()) throw ArgumentError("no shard paths given");
    auto b = std::make_unique<Batcher>(std::move(set.shards), set.vocab, static_cast<int>(seq),
                                       static_cast<int>(batch), (static_cast<uint64_t>(seed_hi) << 32) | seed_lo);
    return static_cast<int32_t>(insert(g.batchers, std::move(b)));
  });
}

int32_t midman_train_evaluate(uint32_t handle, const uint8_t* paths, uint32_t paths_len, uint64_t max_batches) {
  return run([&] {
    Train& t = train_ref(handle);
    Trainer& tr = *t.trainer;
    const ShardSet set = load_shards(paths, paths_len);
    const size_t seq = static_cast<size_t>(tr.seq());
    const size_t global_batch = static_cast<size_t>(tr.batch()) * tr.world();
    const Sequences data(set.shards, static_cast<int>(seq));
    // trainer.rs:218-235: the data must fit the run and the model
    if (!set.shards.empty() && set.vocab != tr.config().vocab)
      throw ArgumentError("the evaluation data has a vocabulary of " + std::to_string(set.vocab) + " and the model " +
                          std::to_string(tr.config().vocab));
    if (set.shards.empty())
      throw ArgumentError("the evaluation data has no vocabulary and the model " + std::to_string(tr.config().vocab));
    if (max_batches == 0 || data.size() == 0) throw ArgumentError("nothing to evaluate");
    // trainer.rs:236-261: batches of the run's size (or all there is), rows at even
    // distances through the sequences; the loss is the mean of the batch losses in f64.
    const size_t batch = std::min(global_batch, data.size());
    const size_t batches = std::min<uint64_t>(max_batches, data.size() / batch);
    const size_t rows = batches * batch;
    const size_t chunk = static_cast<size_t>(tr.batch());  // this rank's capacity in rows
    std::vector<int32_t> in(chunk * seq), tg(chunk * seq);
    double total = 0.0;
    for (size_t b = 0; b < batches; ++b) {
      // a batch larger than one rank's capacity (data parallel) is taken in chunks and
      // recombined as the token-weighted mean of the chunk losses
      double batch_loss = 0.0;
      for (size_t r0 = 0; r0 < batch; r0 += chunk) {
        const size_t n = std::min(chunk, batch - r0);
        for (size_t r = 0; r < n; ++r) {
          const size_t at = static_cast<size_t>((static_cast<unsigned __int128>(b * batch + r0 + r) * data.size()) / rows);
          const uint32_t* w = data.window(at);
          for (size_t j = 0; j < seq; ++j) {
            in[r * seq + j] = static_cast<int32_t>(w[j]);
            tg[r * seq + j] = static_cast<int32_t>(w[j + 1]);
          }
        }
        const float l = tr.eval(in.data(), tg.data(), static_cast<int>(n), static_cast<int>(seq), nullptr);
        batch_loss = n == batch ? static_cast<double>(l) : batch_loss + static_cast<double>(l) * n / batch;
      }
      total += static_cast<double>(static_cast<float>(batch_loss));
    }
    const float loss = static_cast<float>(total / static_cast<double>(batches));
    g.floats.push_back(loss);
    JsonWriter w;
    w.begin_object();
    w.key("loss").number(loss);
    w.key("batches").integer(batches);
    w.key("tokens").integer(rows * seq);
    w.end_object();
    set_text(w.finish());
    return MIDMAN_OK;
  });
}

int32_t midman_batcher_seek(uint32_t handle, uint64_t epoch, uint64_t batches_done) {
  return run([&] {
    Batcher& b = batcher_ref(handle);
    b.seek(epoch, batches_done);
    JsonWriter w;
    w.begin_object();
    write_place(w, b);
    w.end_object();
    set_text(w.finish());
    return MIDMAN_OK;
  });
}

int32_t midman_train_run(uint32_t handle, uint32_t batcher, uint32_t steps) {
  return run([&]() -> int32_t {
    Train& t = train_ref(handle);
    Batcher& b = batcher_ref(batcher);
    Trainer& tr = *t.trainer;
    const int B = tr.batch(), T = tr.seq(), W = tr.world(), r = tr.rank();
    if (b.batch() != static_cast<size_t>(B) * W || b.seq() != static_cast<size_t>(T))
      throw ArgumentError("the batcher gives batches of " + std::to_string(b.batch()) + " x " +
                          std::to_string(b.seq()) + " but the run takes " + std::to_string(B) + " x " +
                          std::to_string(W) + " ranks x " + std::to_string(T));
    const size_t rows = static_cast<size_t>(B) * T;
    std::vector<int32_t> in(rows * W), tg(rows * W);
    std::pair<uint64_t, uint64_t> before[2];
    // Takes the next global batch and prepares this rank's rows in a staging slot;
    // remembers where the batcher was, to put it back if the step fails.
    auto take = [&](int slot) {
      before[slot] = {b.epoch(), b.position()};
      b.next(in.data(), tg.data());
      tr.prepare_batch(in.data() + r * rows, tg.data() + r * rows, B, T, slot);
    };
    auto put_back = [&](int slot) { b.seek(before[slot].first, before[slot].second); };
    if (steps > 0) {
      try {
        take(0);
      } catch (...) {
        put_back(0);
        throw;
      }
      tr.upload_prepared(0, B, T, true);
    }
    for (uint32_t s = 0; s < steps; ++s) {
      const int cur = s & 1, nxt = cur ^ 1;
      const float lr = schedule_lr(t.hyper.max_lr, t.hyper.min_lr, t.hyper.warmup, t.hyper.total, t.step);
      tr.launch_step(lr, adam_of(t.hyper));
      // the host takes and prepares the next batch while the GPU runs this step
      std::exception_ptr next_failed;
      if (s + 1 < steps) {
        try {
          take(nxt);
        } catch (...) {
          next_failed = std::current_exception();
        }
      }
      const StepOut out = tr.collect_step();
      if (record_step(t, out, lr) != MIDMAN_OK) {  // trainer.rs:162-183: nothing of this step stays
        put_back(cur);
        return MIDMAN_STOPPED;
      }
      if (next_failed) {
        put_back(nxt);
        std::rethrow_exception(next_failed);
      }
      if (s + 1 < steps) tr.upload_prepared(nxt, B, T, true);
    }
    JsonWriter w;
    w.begin_object();
    write_place(w, b);
    w.end_object();
    set_text(w.finish());
    return MIDMAN_OK;
  });
}

int32_t midman_batcher_destroy(uint32_t handle) {
  return run([&] {
    if (handle == 0 || handle > g.batchers.size() || !g.batchers[handle - 1])
      throw ArgumentError(std::to_string(handle) + " is not a live batcher handle");
    g.batchers[handle - 1].reset();
    return MIDMAN_OK;
  });
}

int32_t midman_train_destroy(uint32_t handle) {
  return run([&] {
    train_ref(handle);
    g.trains[handle - 1].reset();
    return MIDMAN_OK;
  });
}

}  // extern "C"
