// Internal declarations shared by the oracle's translation units (test
// infrastructure only; see oracle.h).
#pragma once
#include <cmath>
#include <cstdint>
#include <string>
#include <vector>

namespace orc {

// crates/midman-foundation/src/rng.rs:26-119 (xoshiro256** seeded by SplitMix64).
struct Rng {
  uint64_t s[4];
  bool has_spare = false;  // the cached second Box-Muller value (rng.rs:31)
  float spare = 0.0f;
  explicit Rng(uint64_t seed);
  uint64_t next_u64();
  float next_f32();
  double next_f64();
  float uniform(float lo, float hi);
  float normal();
  uint64_t below(uint64_t n);
  template <class T>
  void shuffle(std::vector<T>& items) {
    for (size_t i = items.size(); i-- > 1;) {
      const size_t j = static_cast<size_t>(below(i + 1));
      std::swap(items[i], items[j]);
    }
  }
  Rng fork(uint64_t stream);
};

// crates/midman-model-config/src/config.rs:19-42.
struct Config {
  uint64_t vocab = 0, d_model = 0, n_layers = 0, n_heads = 0, n_kv_heads = 0, d_ff = 0, max_seq_len = 0;
  float rope_theta = 10000.0f, norm_eps = 1e-5f;
  bool tie = true;
  uint64_t head_dim() const { return d_model / n_heads; }
  uint64_t kv_dim() const { return n_kv_heads * head_dim(); }
};
Config config_from(const double* v);
// Empty string when valid, otherwise the offending field (config.rs:106-137).
std::string validate(const Config& c);

struct ParamTensor {
  std::string name;
  std::vector<uint64_t> shape;
  uint64_t offset = 0, numel = 0;
};

// Offsets of one decoder block's tensors in the flat parameter vector.
struct BlockParams {
  uint64_t attn_norm, q, k, v, o, mlp_norm, gate, up, down;
};

struct Model {
  Config cfg;
  std::vector<ParamTensor> tensors;  // MidManModel::parameters order (model.rs:187-197)
  std::vector<BlockParams> blocks;
  uint64_t embed = 0, final_norm = 0, lm_head = 0;
  std::vector<float> params;
  std::vector<float> rope_cos, rope_sin;  // [max_seq_len, head_dim / 2]
};

void build_layout(Model& m);
void init_weights(Model& m, Rng& rng, float std);
void rope_tables(uint64_t head_dim, uint64_t max_seq_len, float theta, std::vector<float>& cos_out,
                 std::vector<float>& sin_out);

// Forward (and optionally backward) of the whole model. probs (optional) receives
// every layer's attention probabilities. Returns 0 or a negative code.
int model_loss(Model& m, const int32_t* inputs, const int32_t* targets, int batch, int seq, float* loss,
               float* grads, std::vector<float>* logits_out, std::vector<float>* probs_out);

// ---- kernels (ops.cpp), crates/midman-tensor/src/kernels.rs:87-109 and ops_*.rs
// C[m,n] += A[m,k] * B[k,n]
void gemm_nn(const float* a, const float* b, float* c, size_t m, size_t k, size_t n);
// C[m,n] += A[m,k] * B[n,k]^T  (via a transposed copy of B, kernels.rs:66-75)
void gemm_nt(const float* a, const float* b, float* c, size_t m, size_t k, size_t n);
// C[m,n] += A[k,m]^T * B[k,n]
void gemm_tn(const float* a, const float* b, float* c, size_t k, size_t m, size_t n);
// One thread: C(i, j) += sum_p A(i, p) * B[p][j] with A(i, p) = a[i * rs + p * cs],
// B row stride ldb, C row stride ldc; the same per-element order as gemm_nn.
void gemm_strided_serial(const float* a, size_t rs, size_t cs, const float* b, size_t ldb, float* c, size_t ldc,
                         size_t m, size_t k, size_t n);

void set_threads(int n);

// Known-answer entry points (or_model.cpp).
void causal_attention(const Config& c, const float* q, const float* k, const float* v, size_t B, size_t T,
                      float* out, float* probs);
void softmax_rows(const float* x, float* y, size_t rows, size_t cols);
float cross_entropy(const float* logits, const int32_t* targets, size_t n, size_t v, float* grad);
void rms_norm_layer(const float* x, const float* w, size_t rows, size_t d, float eps, float* y, float* rstd_out);
void rms_norm_layer_bwd(const float* x, const float* w, const float* gy, size_t rows, size_t d, float eps, float* dx,
                        float* dw);
void rope_layer(float* x, size_t BH, size_t T, size_t hd, const float* cos_t, const float* sin_t, bool backward);
void swiglu_layer(const float* g, const float* u, size_t n, float* act, const float* dact, float* dg, float* du);
void embedding_layer(const int32_t* ids, size_t rows, const float* table, size_t d, float* out, const float* dx,
                     float* dtable);

// One AdamW update over a flat array (adamw.rs:192-215); decay: the parameter has rank >= 2.
void adamw_update(float* x, const float* g, float* m, float* v, size_t n, bool decay, uint64_t step, float lr,
                  float beta1, float beta2, float eps, float weight_decay);

}  // namespace orc
