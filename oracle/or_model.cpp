// Oracle part 3: MidManModel forward and backward, written out op by op in the
// order the reference's autograd tape records and replays them.
// Test infrastructure only (see oracle.h).
#include <omp.h>

#include <cmath>
#include <cstring>
#include <limits>
#include <vector>

#include "oracle_internal.h"

namespace orc {

namespace {

using Vec = std::vector<float>;

// rms_norm (crates/midman-nn/src/norm.rs:21-39) built from primitives:
// sq = x*x; ms = mean_axis(-1) = sum_axis * (1/len); t = ms + eps; inv = t^-0.5;
// y1 = x*inv; y = y1*w.
struct NormSaved {
  Vec t;   // [rows]
  Vec inv; // [rows]
  Vec y1;  // [rows, d]
};

void rms_norm_fwd(const float* x, const float* w, size_t rows, size_t d, float eps, float* y, NormSaved& s) {
  s.t.resize(rows);
  s.inv.resize(rows);
  s.y1.resize(rows * d);
  const float factor = 1.0f / static_cast<float>(d);  // ops_reduce.rs:87-90 mean_axis
#pragma omp parallel for schedule(static) if (rows * d > (1u << 15))
  for (long long r = 0; r < static_cast<long long>(rows); ++r) {
    const float* xr = x + r * d;
    float total = 0.0f;  // sum_axis contiguous path (ops_reduce.rs:40-47)
    for (size_t j = 0; j < d; ++j) total += xr[j] * xr[j];
    const float ms = total * factor;
    const float t = ms + eps;
    const float inv = std::pow(t, -0.5f);
    s.t[r] = t;
    s.inv[r] = inv;
    for (size_t j = 0; j < d; ++j) {
      const float v1 = xr[j] * inv;
      s.y1[r * d + j] = v1;
      y[r * d + j] = v1 * w[j];
    }
  }
}

// Backward of the same primitive chain: each op's closure from ops_elementwise.rs
// (mul: g*other, powf: g * p * x^(p-1), scale: g*factor) and ops_reduce.rs (sum_axis
// fills the row); the weight's gradient is summed over rows (shape.rs:208 sum_to_shape).
void rms_norm_bwd(const float* x, const float* w, const NormSaved& s, const float* gy, size_t rows, size_t d,
                  float* dx /* accumulated into */, float* dw /* accumulated into */) {
  const float factor = 1.0f / static_cast<float>(d);
  std::vector<float> dw_local(d, 0.0f);
  // The weight gradient: sum over rows in row order (sum_to_shape keeps the last axis).
  for (size_t r = 0; r < rows; ++r)
    for (size_t j = 0; j < d; ++j) dw_local[j] += gy[r * d + j] * s.y1[r * d + j];
  for (size_t j = 0; j < d; ++j) dw[j] += dw_local[j];
#pragma omp parallel for schedule(static) if (rows * d > (1u << 15))
  for (long long r = 0; r < static_cast<long long>(rows); ++r) {
    const float* xr = x + r * d;
    const float* gr = gy + r * d;
    float dinv = 0.0f;
    for (size_t j = 0; j < d; ++j) dinv += (gr[j] * w[j]) * xr[j];
    const float dt = dinv * (-0.5f * std::pow(s.t[r], -0.5f - 1.0f));
    const float dsum = dt * factor;
    for (size_t j = 0; j < d; ++j) {
      const float dy1 = gr[j] * w[j];
      const float a = dy1 * s.inv[r];
      const float b = dsum * xr[j];
      dx[r * d + j] += (a + b) + b;
    }
  }
}

float sigmoid(float x) { return 1.0f / (1.0f + std::exp(-x)); }

// [B, T, heads, hd] (token-major projection) -> [B, heads, T, hd] (permute copy).
void split_heads(const float* proj, size_t B, size_t T, size_t heads, size_t hd, float* out) {
  for (size_t b = 0; b < B; ++b)
    for (size_t t = 0; t < T; ++t)
      for (size_t h = 0; h < heads; ++h)
        std::memcpy(out + ((b * heads + h) * T + t) * hd, proj + ((b * T + t) * heads + h) * hd, hd * sizeof(float));
}

void merge_heads(const float* heads_, size_t B, size_t T, size_t H, size_t hd, float* out) {
  for (size_t b = 0; b < B; ++b)
    for (size_t t = 0; t < T; ++t)
      for (size_t h = 0; h < H; ++h)
        std::memcpy(out + ((b * T + t) * H + h) * hd, heads_ + ((b * H + h) * T + t) * hd, hd * sizeof(float));
}

// apply_rope (rope.rs:20-33) on [B, heads, T, hd]: first = x1*cos - x2*sin, second = x2*cos + x1*sin.
void rope_fwd(float* x, size_t BH, size_t T, size_t hd, const float* cos_t, const float* sin_t) {
  const size_t half = hd / 2;
  for (size_t bh = 0; bh < BH; ++bh)
    for (size_t t = 0; t < T; ++t) {
      float* v = x + (bh * T + t) * hd;
      const float* c = cos_t + t * half;
      const float* s = sin_t + t * half;
      for (size_t i = 0; i < half; ++i) {
        const float x1 = v[i], x2 = v[i + half];
        v[i] = x1 * c[i] - x2 * s[i];
        v[i + half] = x2 * c[i] + x1 * s[i];
      }
    }
}

// Gradient of rope_fwd through concat, sub/add and the broadcast products.
void rope_bwd(float* g, size_t BH, size_t T, size_t hd, const float* cos_t, const float* sin_t) {
  const size_t half = hd / 2;
  for (size_t bh = 0; bh < BH; ++bh)
    for (size_t t = 0; t < T; ++t) {
      float* v = g + (bh * T + t) * hd;
      const float* c = cos_t + t * half;
      const float* s = sin_t + t * half;
      for (size_t i = 0; i < half; ++i) {
        const float g1 = v[i], g2 = v[i + half];
        v[i] = g1 * c[i] + g2 * s[i];
        v[i + half] = g2 * c[i] + (-g1) * s[i];
      }
    }
}

struct LayerSaved {
  Vec x;        // block input [N, D]
  NormSaved n1;
  Vec xn1;      // [N, D]
  Vec q, k, v;  // [B, H, T, hd] after rope; [B, Hkv, T, hd] after rope; [B, Hkv, T, hd]
  Vec probs;    // [B, H, T, T]
  Vec merged;   // [N, D]
  Vec h;        // [N, D]
  NormSaved n2;
  Vec xn2;      // [N, D]
  Vec gate, gs, up, act;  // [N, F]
};


// causal_attention_weights + probs.matmul(v) (attention.rs:79-85, :160-166) for one
// layer: repeat_interleave for grouped heads, k^T copy, batched gemm_nn, scale,
// + causal_mask (-1e9 above the diagonal), softmax (ops_reduce.rs:97-126), P v.
void attention_fwd(const Config& c, size_t B, size_t T, LayerSaved& L, Vec& context) {
  const size_t H = c.n_heads, Hkv = c.n_kv_heads, hd = c.head_dim(), groups = H / Hkv;
  const float scale = 1.0f / std::sqrt(static_cast<float>(hd));
  L.probs.assign(B * H * T * T, 0.0f);
  context.assign(B * H * T * hd, 0.0f);
#pragma omp parallel for schedule(dynamic)
  for (long long bh = 0; bh < static_cast<long long>(B * H); ++bh) {
    const size_t b = bh / H, h = bh % H, hk = h / groups;
    const float* q = L.q.data() + bh * T * hd;
    const float* k = L.k.data() + (b * Hkv + hk) * T * hd;
    const float* v = L.v.data() + (b * Hkv + hk) * T * hd;
    std::vector<float> kt(hd * T), s(T * T, 0.0f);
    for (size_t j = 0; j < T; ++j)
      for (size_t p = 0; p < hd; ++p) kt[p * T + j] = k[j * hd + p];
    // s[i][j] += q[i][p] * kt[p][j], p ascending
    gemm_strided_serial(q, hd, 1, kt.data(), T, s.data(), T, T, hd, T);
    float* y = L.probs.data() + bh * T * T;
    for (size_t i = 0; i < T; ++i) {
      float* row = s.data() + i * T;
      for (size_t j = 0; j < T; ++j) row[j] = row[j] * scale + (j > i ? -1.0e9f : 0.0f);
      float mx = -std::numeric_limits<float>::infinity();
      for (size_t j = 0; j < T; ++j) mx = std::fmax(mx, row[j]);
      float sum = 0.0f;
      for (size_t j = 0; j < T; ++j) {
        const float e = std::exp(row[j] - mx);
        y[i * T + j] = e;
        sum += e;
      }
      const float inv = 1.0f / sum;
      for (size_t j = 0; j < T; ++j) y[i * T + j] *= inv;
    }
    float* ctx = context.data() + bh * T * hd;
    // ctx[i][p] += y[i][j] * v[j][p], j ascending
    gemm_strided_serial(y, T, 1, v, hd, ctx, hd, T, T, hd);
  }
}

// Backward of attention_fwd: matmul closures (ops_matmul.rs:100-125: gemm_nt for the
// left operand, gemm_tn for the right), softmax y*(g - sum(g*y)) (ops_reduce.rs:131-142),
// scale, transpose, and repeat_interleave summing each group's copies in order
// (ops_shape.rs:204-217). Returns dq [B,H,T,hd], dk and dv [B,Hkv,T,hd].
void attention_bwd(const Config& c, size_t B, size_t T, const LayerSaved& L, const Vec& dctx, Vec& dq, Vec& dk,
                   Vec& dv) {
  const size_t H = c.n_heads, Hkv = c.n_kv_heads, hd = c.head_dim(), groups = H / Hkv;
  const float scale = 1.0f / std::sqrt(static_cast<float>(hd));
  dq.assign(B * H * T * hd, 0.0f);
  Vec dk_e(B * H * T * hd, 0.0f), dv_e(B * H * T * hd, 0.0f);
#pragma omp parallel for schedule(dynamic)
  for (long long bh = 0; bh < static_cast<long long>(B * H); ++bh) {
    const size_t b = bh / H, h = bh % H, hk = h / groups;
    const float* q = L.q.data() + bh * T * hd;
    const float* k = L.k.data() + (b * Hkv + hk) * T * hd;
    const float* v = L.v.data() + (b * Hkv + hk) * T * hd;
    const float* y = L.probs.data() + bh * T * T;
    const float* g = dctx.data() + bh * T * hd;
    std::vector<float> dp(T * T, 0.0f), ds(T * T, 0.0f);
    // dprobs = gemm_nt(g, v): dot-product form over hd
    // (as gemm_nn of g and a transposed copy of v: p ascending from zero per element)
    std::vector<float> vt(hd * T);
    for (size_t j = 0; j < T; ++j)
      for (size_t p = 0; p < hd; ++p) vt[p * T + j] = v[j * hd + p];
    gemm_strided_serial(g, hd, 1, vt.data(), T, dp.data(), T, T, hd, T);
    // dv_expanded = gemm_tn(probs, g)
    float* dve = dv_e.data() + bh * T * hd;
    // dve[j][p] += y[i][j] * g[i][p], i ascending
    gemm_strided_serial(y, 1, T, g, hd, dve, hd, T, T, hd);
    // softmax backward, then the scale
    for (size_t i = 0; i < T; ++i) {
      float dot = 0.0f;
      for (size_t j = 0; j < T; ++j) dot += dp[i * T + j] * y[i * T + j];
      for (size_t j = 0; j < T; ++j) ds[i * T + j] = (y[i * T + j] * (dp[i * T + j] - dot)) * scale;
    }
    // dq = gemm_nt(ds, k^T) = ds k (dot-product form over j)
    float* dqo = dq.data() + bh * T * hd;
    // dq[i][p] = sum of ds[i][j] * k[j][p], j ascending from zero
    gemm_strided_serial(ds.data(), T, 1, k, hd, dqo, hd, T, T, hd);
    // dk^T = gemm_tn(q, ds): dkt[p][j] = sum_i q[i][p] ds[i][j]; transposed back
    float* dke = dk_e.data() + bh * T * hd;
    // dke[j][p] += ds[i][j] * q[i][p], i ascending
    gemm_strided_serial(ds.data(), 1, T, q, hd, dke, hd, T, T, hd);
  }
  dk.assign(B * Hkv * T * hd, 0.0f);
  dv.assign(B * Hkv * T * hd, 0.0f);
  for (size_t b = 0; b < B; ++b)
    for (size_t hk = 0; hk < Hkv; ++hk)
      for (size_t r = 0; r < groups; ++r) {
        const size_t h = hk * groups + r;
        const float* sk = dk_e.data() + (b * H + h) * T * hd;
        const float* sv = dv_e.data() + (b * H + h) * T * hd;
        float* tk = dk.data() + (b * Hkv + hk) * T * hd;
        float* tv = dv.data() + (b * Hkv + hk) * T * hd;
        for (size_t e = 0; e < T * hd; ++e) {
          tk[e] += sk[e];
          tv[e] += sv[e];
        }
      }
}

}  // namespace

// MidManModel::loss (model.rs:127-183) and, with grads, Tensor::backward of it.
int model_loss(Model& m, const int32_t* inputs, const int32_t* targets, int batch, int seq, float* loss,
               float* grads, std::vector<float>* logits_out, std::vector<float>* probs_out) {
  const Config& c = m.cfg;
  if (batch <= 0 || seq <= 0) return -1;
  if (static_cast<uint64_t>(seq) > c.max_seq_len) return -1;
  const size_t B = batch, T = seq, N = B * T, D = c.d_model, F = c.d_ff, V = c.vocab;
  const size_t H = c.n_heads, Hkv = c.n_kv_heads, hd = c.head_dim(), KV = c.kv_dim();
  for (size_t i = 0; i < N; ++i) {
    if (inputs[i] < 0 || static_cast<uint64_t>(inputs[i]) >= V) return -4;
    if (targets && (targets[i] < 0 || static_cast<uint64_t>(targets[i]) >= V)) return -4;
  }
  const float* P = m.params.data();
  const float eps = c.norm_eps;

  // embedding gather (ops_shape.rs:230-255)
  Vec x(N * D);
  for (size_t r = 0; r < N; ++r) std::memcpy(&x[r * D], P + m.embed + inputs[r] * D, D * sizeof(float));

  std::vector<LayerSaved> saved(c.n_layers);
  if (probs_out) probs_out->clear();
  Vec proj, context;
  for (size_t l = 0; l < c.n_layers; ++l) {
    const BlockParams& bp = m.blocks[l];
    LayerSaved& L = saved[l];
    L.x = x;
    L.xn1.resize(N * D);
    rms_norm_fwd(x.data(), P + bp.attn_norm, N, D, eps, L.xn1.data(), L.n1);
    // q, k, v projections -> [B, heads, T, hd] (attention.rs:157-160)
    proj.assign(N * D, 0.0f);
    gemm_nn(L.xn1.data(), P + bp.q, proj.data(), N, D, D);
    L.q.resize(N * D);
    split_heads(proj.data(), B, T, H, hd, L.q.data());
    rope_fwd(L.q.data(), B * H, T, hd, m.rope_cos.data(), m.rope_sin.data());
    proj.assign(N * KV, 0.0f);
    gemm_nn(L.xn1.data(), P + bp.k, proj.data(), N, D, KV);
    L.k.resize(N * KV);
    split_heads(proj.data(), B, T, Hkv, hd, L.k.data());
    rope_fwd(L.k.data(), B * Hkv, T, hd, m.rope_cos.data(), m.rope_sin.data());
    proj.assign(N * KV, 0.0f);
    gemm_nn(L.xn1.data(), P + bp.v, proj.data(), N, D, KV);
    L.v.resize(N * KV);
    split_heads(proj.data(), B, T, Hkv, hd, L.v.data());
    attention_fwd(c, B, T, L, context);
    if (probs_out) probs_out->insert(probs_out->end(), L.probs.begin(), L.probs.end());
    L.merged.resize(N * D);
    merge_heads(context.data(), B, T, H, hd, L.merged.data());
    // h = x + merged Wo (block.rs:78-79)
    Vec attended(N * D, 0.0f);
    gemm_nn(L.merged.data(), P + bp.o, attended.data(), N, D, D);
    L.h.resize(N * D);
    for (size_t i = 0; i < N * D; ++i) L.h[i] = x[i] + attended[i];
    // swiglu (mlp.rs:20-24): silu(x Wg) * (x Wu) Wd
    L.xn2.resize(N * D);
    rms_norm_fwd(L.h.data(), P + bp.mlp_norm, N, D, eps, L.xn2.data(), L.n2);
    L.gate.assign(N * F, 0.0f);
    gemm_nn(L.xn2.data(), P + bp.gate, L.gate.data(), N, D, F);
    L.gs.resize(N * F);
    for (size_t i = 0; i < N * F; ++i) L.gs[i] = L.gate[i] * sigmoid(L.gate[i]);  // ops_elementwise.rs:355-364
    L.up.assign(N * F, 0.0f);
    gemm_nn(L.xn2.data(), P + bp.up, L.up.data(), N, D, F);
    L.act.resize(N * F);
    for (size_t i = 0; i < N * F; ++i) L.act[i] = L.gs[i] * L.up[i];
    Vec down(N * D, 0.0f);
    gemm_nn(L.act.data(), P + bp.down, down.data(), N, F, D);
    for (size_t i = 0; i < N * D; ++i) x[i] = L.h[i] + down[i];
  }
  // final norm and the head (model.rs:160-164): tied = x E^T through a transposed copy
  NormSaved nf;
  Vec xf(N * D);
  rms_norm_fwd(x.data(), P + m.final_norm, N, D, eps, xf.data(), nf);
  Vec head_t;  // [D, V]
  const float* head;
  if (c.tie) {
    head_t.resize(D * V);
#pragma omp parallel for schedule(static)
    for (long long d = 0; d < static_cast<long long>(D); ++d)
      for (size_t v = 0; v < V; ++v) head_t[d * V + v] = P[m.embed + v * D + d];
    head = head_t.data();
  } else {
    head = P + m.lm_head;
  }
  Vec logits(N * V, 0.0f);
  gemm_nn(xf.data(), head, logits.data(), N, D, V);
  if (logits_out) *logits_out = logits;
  if (!targets) return 0;

  // cross_entropy (ops_reduce.rs:236-276): loss total in f64, recomputed max/sum in backward
  double total = 0.0;
  for (size_t r = 0; r < N; ++r) {
    const float* row = &logits[r * V];
    float mx = -std::numeric_limits<float>::infinity();
    for (size_t j = 0; j < V; ++j) mx = std::fmax(mx, row[j]);
    float sum = 0.0f;
    for (size_t j = 0; j < V; ++j) sum += std::exp(row[j] - mx);
    total += static_cast<double>(mx + std::log(sum) - row[targets[r]]);
  }
  *loss = static_cast<float>(total / static_cast<double>(N));
  if (!grads) return 0;

  std::memset(grads, 0, m.params.size() * sizeof(float));
  const float scale = 1.0f / static_cast<float>(N);
  Vec g(N * V);  // d loss / d logits
#pragma omp parallel for schedule(static)
  for (long long r = 0; r < static_cast<long long>(N); ++r) {
    const float* row = &logits[r * V];
    float* drow = &g[r * V];
    float mx = -std::numeric_limits<float>::infinity();
    for (size_t j = 0; j < V; ++j) mx = std::fmax(mx, row[j]);
    float sum = 0.0f;
    for (size_t j = 0; j < V; ++j) sum += std::exp(row[j] - mx);
    for (size_t j = 0; j < V; ++j) drow[j] = std::exp(row[j] - mx) / sum * scale;
    drow[targets[r]] -= scale;
  }
  // head matmul backward (ops_matmul.rs:62-74)
  Vec dxf(N * D, 0.0f);
  gemm_nt(g.data(), head, dxf.data(), N, V, D);
  if (c.tie) {
    Vec dhead_t(D * V, 0.0f);
    gemm_tn(xf.data(), g.data(), dhead_t.data(), N, D, V);
#pragma omp parallel for schedule(static)
    for (long long v = 0; v < static_cast<long long>(V); ++v)
      for (size_t d = 0; d < D; ++d) grads[m.embed + v * D + d] = dhead_t[d * V + v];
  } else {
    gemm_tn(xf.data(), g.data(), grads + m.lm_head, N, D, V);
  }
  g = Vec();
  Vec dx(N * D, 0.0f);
  rms_norm_bwd(x.data(), P + m.final_norm, nf, dxf.data(), N, D, dx.data(), grads + m.final_norm);

  Vec dxn(N * D), dact(N * F), dgs(N * F), dup(N * F), dgate(N * F), dmerged(N * D), dctx(N * D);
  Vec dq, dk, dv, dproj;
  for (size_t li = c.n_layers; li-- > 0;) {
    const BlockParams& bp = m.blocks[li];
    LayerSaved& L = saved[li];
    // out = h + down: dh = dx, ddown = dx
    Vec& dh = dx;  // dx currently holds d out
    std::fill(dact.begin(), dact.end(), 0.0f);
    gemm_nt(dx.data(), P + bp.down, dact.data(), N, D, F);
    gemm_tn(L.act.data(), dx.data(), grads + bp.down, N, F, D);
    for (size_t i = 0; i < N * F; ++i) {
      dgs[i] = dact[i] * L.up[i];
      dup[i] = dact[i] * L.gs[i];
      const float s = sigmoid(L.gate[i]);
      dgate[i] = dgs[i] * (s * (1.0f + L.gate[i] * (1.0f - s)));
    }
    std::fill(dxn.begin(), dxn.end(), 0.0f);
    gemm_nt(dup.data(), P + bp.up, dxn.data(), N, F, D);
    gemm_tn(L.xn2.data(), dup.data(), grads + bp.up, N, D, F);
    Vec dxn_g(N * D, 0.0f);
    gemm_nt(dgate.data(), P + bp.gate, dxn_g.data(), N, F, D);
    gemm_tn(L.xn2.data(), dgate.data(), grads + bp.gate, N, D, F);
    for (size_t i = 0; i < N * D; ++i) dxn[i] += dxn_g[i];
    rms_norm_bwd(L.h.data(), P + bp.mlp_norm, L.n2, dxn.data(), N, D, dh.data(), grads + bp.mlp_norm);
    // h = x + attended: dattended = dh; d x = dh (kept in dx)
    std::fill(dmerged.begin(), dmerged.end(), 0.0f);
    gemm_nt(dh.data(), P + bp.o, dmerged.data(), N, D, D);
    gemm_tn(L.merged.data(), dh.data(), grads + bp.o, N, D, D);
    split_heads(dmerged.data(), B, T, H, hd, dctx.data());
    attention_bwd(c, B, T, L, dctx, dq, dk, dv);
    rope_bwd(dq.data(), B * H, T, hd, m.rope_cos.data(), m.rope_sin.data());
    rope_bwd(dk.data(), B * Hkv, T, hd, m.rope_cos.data(), m.rope_sin.data());
    std::fill(dxn.begin(), dxn.end(), 0.0f);
    dproj.resize(N * D);
    merge_heads(dq.data(), B, T, H, hd, dproj.data());
    gemm_nt(dproj.data(), P + bp.q, dxn.data(), N, D, D);
    gemm_tn(L.xn1.data(), dproj.data(), grads + bp.q, N, D, D);
    dproj.resize(N * KV);
    // each projection's input gradient is its own product, then summed (autograd.rs:44-56)
    Vec part(N * D);
    merge_heads(dk.data(), B, T, Hkv, hd, dproj.data());
    std::fill(part.begin(), part.end(), 0.0f);
    gemm_nt(dproj.data(), P + bp.k, part.data(), N, KV, D);
    for (size_t i = 0; i < N * D; ++i) dxn[i] += part[i];
    gemm_tn(L.xn1.data(), dproj.data(), grads + bp.k, N, D, KV);
    merge_heads(dv.data(), B, T, Hkv, hd, dproj.data());
    std::fill(part.begin(), part.end(), 0.0f);
    gemm_nt(dproj.data(), P + bp.v, part.data(), N, KV, D);
    for (size_t i = 0; i < N * D; ++i) dxn[i] += part[i];
    gemm_tn(L.xn1.data(), dproj.data(), grads + bp.v, N, D, KV);
    rms_norm_bwd(L.x.data(), P + bp.attn_norm, L.n1, dxn.data(), N, D, dx.data(), grads + bp.attn_norm);
    L = LayerSaved();
  }
  // embedding scatter-add (ops_shape.rs:262-272), added after the head's share
  for (size_t r = 0; r < N; ++r) {
    float* t = grads + m.embed + inputs[r] * D;
    for (size_t d = 0; d < D; ++d) t[d] += dx[r * D + d];
  }
  return 0;
}

}  // namespace orc

namespace orc {

// Stand-alone entry points for the known-answer tests: the same code paths the
// model uses, on caller-provided arrays.
void causal_attention(const Config& c, const float* q, const float* k, const float* v, size_t B, size_t T,
                      float* out, float* probs) {
  LayerSaved L;
  const size_t H = c.n_heads, Hkv = c.n_kv_heads, hd = c.head_dim();
  L.q.assign(q, q + B * H * T * hd);
  L.k.assign(k, k + B * Hkv * T * hd);
  L.v.assign(v, v + B * Hkv * T * hd);
  Vec ctx;
  attention_fwd(c, B, T, L, ctx);
  std::memcpy(out, ctx.data(), ctx.size() * sizeof(float));
  if (probs) std::memcpy(probs, L.probs.data(), L.probs.size() * sizeof(float));
}

// ops_reduce.rs:97-126, contiguous-axis path.
void softmax_rows(const float* x, float* y, size_t rows, size_t cols) {
  for (size_t r = 0; r < rows; ++r) {
    const float* row = x + r * cols;
    float* dst = y + r * cols;
    float mx = -std::numeric_limits<float>::infinity();
    for (size_t j = 0; j < cols; ++j) mx = std::fmax(mx, row[j]);
    float sum = 0.0f;
    for (size_t j = 0; j < cols; ++j) {
      const float e = std::exp(row[j] - mx);
      dst[j] = e;
      sum += e;
    }
    const float inv = 1.0f / sum;
    for (size_t j = 0; j < cols; ++j) dst[j] *= inv;
  }
}

// ops_reduce.rs:236-276: mean loss (f64 total) and, if grad != null, d loss / d logits.
// Known-answer entry points of single layers, for the kernel-level tests.
// rms_norm (norm.rs:21-39); rstd_out[r] = the row's t^-0.5.
void rms_norm_layer(const float* x, const float* w, size_t rows, size_t d, float eps, float* y, float* rstd_out) {
  NormSaved s;
  rms_norm_fwd(x, w, rows, d, eps, y, s);
  if (rstd_out) std::memcpy(rstd_out, s.inv.data(), rows * sizeof(float));
}

// Backward of rms_norm (the six primitives' closures): dx, dw overwritten.
void rms_norm_layer_bwd(const float* x, const float* w, const float* gy, size_t rows, size_t d, float eps, float* dx,
                        float* dw) {
  NormSaved s;
  Vec y(rows * d);
  rms_norm_fwd(x, w, rows, d, eps, y.data(), s);
  std::memset(dx, 0, rows * d * sizeof(float));
  std::memset(dw, 0, d * sizeof(float));
  rms_norm_bwd(x, w, s, gy, rows, d, dx, dw);
}

// apply_rope (rope.rs:20-33) or its gradient, in place on [B, heads, T, hd].
void rope_layer(float* x, size_t BH, size_t T, size_t hd, const float* cos_t, const float* sin_t, bool backward) {
  if (backward)
    rope_bwd(x, BH, T, hd, cos_t, sin_t);
  else
    rope_fwd(x, BH, T, hd, cos_t, sin_t);
}

// swiglu (mlp.rs:20-24): act = silu(g) * u; with dact, the gradients dg, du.
void swiglu_layer(const float* g, const float* u, size_t n, float* act, const float* dact, float* dg, float* du) {
  for (size_t i = 0; i < n; ++i) {
    const float gs = g[i] * sigmoid(g[i]);
    if (act) act[i] = gs * u[i];
    if (dact) {
      const float dgs = dact[i] * u[i];
      du[i] = dact[i] * gs;
      const float sg = sigmoid(g[i]);
      dg[i] = dgs * (sg * (1.0f + g[i] * (1.0f - sg)));
    }
  }
}

// embedding gather (ops_shape.rs:230-255) and scatter-add (:262-272, rows in order).
void embedding_layer(const int32_t* ids, size_t rows, const float* table, size_t d, float* out, const float* dx,
                     float* dtable) {
  for (size_t r = 0; r < rows; ++r) {
    if (out) std::memcpy(out + r * d, table + static_cast<size_t>(ids[r]) * d, d * sizeof(float));
    if (dx)
      for (size_t j = 0; j < d; ++j) dtable[static_cast<size_t>(ids[r]) * d + j] += dx[r * d + j];
  }
}

float cross_entropy(const float* logits, const int32_t* targets, size_t n, size_t v, float* grad) {
  double total = 0.0;
  const float scale = 1.0f / static_cast<float>(n);
  for (size_t r = 0; r < n; ++r) {
    const float* row = logits + r * v;
    float mx = -std::numeric_limits<float>::infinity();
    for (size_t j = 0; j < v; ++j) mx = std::fmax(mx, row[j]);
    float sum = 0.0f;
    for (size_t j = 0; j < v; ++j) sum += std::exp(row[j] - mx);
    total += static_cast<double>(mx + std::log(sum) - row[targets[r]]);
    if (grad) {
      for (size_t j = 0; j < v; ++j) grad[r * v + j] = std::exp(row[j] - mx) / sum * scale;
      grad[r * v + targets[r]] -= scale;
    }
  }
  return static_cast<float>(total / static_cast<double>(n));
}

}  // namespace orc
