// Causal grouped-query attention on the TF32 tensor cores: the score and
// probability matrices of every (batch, head) are formed by the batched tcgen05
// GEMM (gemm.cu) restricted to the causal part, with the softmax and its
// backward as row kernels between them.
//
// Forward (attention.rs:79-102):  S = Q K^T  ->  P = softmax(S * scale + mask), lse  ->  O = P V
// Backward (autograd of the same):  S, dP = dO V^T  ->  P, dS = P * (dP - delta) * scale
//   ->  dV = P^T dO,  dK = dS^T Q,  dQ = dS K
// S/P and dP/dS live in [B*H, T, ldS] buffers. Only the lower-triangular part
// is computed: output tiles above the diagonal are skipped and the K loops stop
// (or start) at the diagonal block, so for causal T x T products about half the
// work of the dense product is done. Entries of a row past the query position but
// inside its 128-wide block are written as exact zeros, which is what a product
// whose K loop runs to the end of that block reads. K and V are addressed per
// key/value head (no copies for grouped-query sharing); with groups > 1 the
// per-query-head dK and dV are summed over each group afterwards.
#include <cuda_runtime.h>

#include <cmath>
#include <stdexcept>
#include <string>

#include "attention.h"
#include "device.h"
#include "gemm.h"

namespace mm {

namespace {

constexpr int kRowBlock = 128;  // the GEMM's BM: rows share their causal K range per 128-row block

void check(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

void check_gemm(int rc, const char* what) {
  if (rc) throw std::runtime_error(std::string(what) + ": " + gemm_status_string(rc));
}

__device__ __forceinline__ int row_end(int i, int T) { return min(T, (i / kRowBlock + 1) * kRowBlock); }

// One warp per score row (b, h, i): P = softmax over j <= i of S * scale, zeros
// for i < j < row_end, lse = max + log(sum) (ops_reduce.rs:97-126 with the mask
// of attention.rs:24-27 folded in).
__global__ void softmax_rows_kernel(float* __restrict__ S, long long ldS, int T, long long rows, float scale,
                                    float* __restrict__ lse) {
  const long long r = (blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x) / 32;
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  const int i = static_cast<int>(r % T);
  float* row = S + r * ldS;
  const int n = i + 1, end = row_end(i, T);
  float m = -INFINITY;
  for (int j = lane; j < n; j += 32) m = fmaxf(m, row[j] * scale);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  float s = 0.0f;
  for (int j = lane; j < n; j += 32) s += expf(row[j] * scale - m);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float inv = 1.0f / s;
  for (int j = lane; j < end; j += 32) row[j] = j < n ? expf(row[j] * scale - m) * inv : 0.0f;
  if (lane == 0) lse[r] = m + logf(s);
}

// One warp per row: P = exp(S * scale - lse) and dS = P * (dP - delta) * scale
// (the softmax backward, ops_reduce.rs:131-142, then the score scale), written
// over S and dP.
__global__ void softmax_bwd_rows_kernel(float* __restrict__ S, float* __restrict__ dP, long long ldS, int T,
                                        long long rows, float scale, const float* __restrict__ lse,
                                        const float* __restrict__ delta) {
  const long long r = (blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x) / 32;
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  const int i = static_cast<int>(r % T);
  float* srow = S + r * ldS;
  float* drow = dP + r * ldS;
  const float l = lse[r], dl = delta[r];
  const int end = row_end(i, T);
  for (int j = lane; j < end; j += 32) {
    float p = 0.0f, ds = 0.0f;
    if (j <= i) {
      p = expf(srow[j] * scale - l);
      ds = (p * (drow[j] - dl)) * scale;
    }
    srow[j] = p;
    drow[j] = ds;
  }
}

// dst[b, t, hk, :] = sum over the group's query heads of src[b, t, hk*G + g, :].
__global__ void group_sum_kernel(const float* __restrict__ src, float* __restrict__ dst, long long tokens, int Hkv,
                                 int G, int hd) {
  const long long total = tokens * Hkv * hd;
  for (long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int d = static_cast<int>(idx % hd);
    const long long th = idx / hd;
    const int hk = static_cast<int>(th % Hkv);
    const long long t = th / Hkv;
    const float* s = src + (t * Hkv * G + static_cast<long long>(hk) * G) * hd + d;
    float acc = 0.0f;
    for (int g = 0; g < G; ++g) acc += s[static_cast<long long>(g) * hd];
    dst[idx] = acc;
  }
}

int blocks_for(long long threads) {
  long long b = (threads + 255) / 256;
  return static_cast<int>(b < 1 ? 1 : b);
}

// Views of the operands (extents and strides in elements).
BatchedOperand heads_view(const float* p, bool mn, const AttnShape& s, long long ld, int heads, int group) {
  // token-major [B, T, heads, hd]: inner = hd, rows = T
  return BatchedOperand{p, mn, s.hd, heads, s.T, s.B, s.hd, ld, static_cast<long long>(s.T) * ld, s.H, group};
}

BatchedOperand scores_view(const float* p, bool mn, const AttnShape& s, long long ldS) {
  // [B*H, T, ldS]: inner = keys, rows = queries, one matrix per (b, h) as the
  // view's batch index (its head dimension has extent 1)
  const long long bh = static_cast<long long>(s.B) * s.H;
  return BatchedOperand{p, mn, s.T, 1, s.T, bh, ldS, ldS, static_cast<long long>(s.T) * ldS, 1, 1};
}

int tile_for(int hd) { return hd <= 64 ? 64 : 128; }

}  // namespace

long long attention_scores_ld(int T) { return (T + 3) & ~3ll; }

bool attention_tc_supported(const AttnShape& s) {
  return (s.hd == 32 || s.hd == 64 || s.hd == 128) && s.H % s.Hkv == 0 && s.ldq % 4 == 0 && s.ldk % 4 == 0 &&
         s.ldv % 4 == 0 && s.ldo % 4 == 0;
}

void attention_forward_tc(const AttnShape& s, const float* q, const float* k, const float* v, float* o, float* lse,
                          float* S, cudaStream_t stream) {
  attention_forward_tc(s, q, k, v, o, lse, S, device_context().d_err, stream);
}

void attention_forward_tc(const AttnShape& s, const float* q, const float* k, const float* v, float* o, float* lse,
                          float* S, int* d_err, cudaStream_t stream) {
  const int G = s.H / s.Hkv;
  const int BH = s.B * s.H;
  const long long ldS = attention_scores_ld(s.T);
  // S = Q K^T, tiles above the diagonal skipped
  GemmBatch bs;
  bs.c_zdiv = BH;
  bs.c_sh = static_cast<long long>(s.T) * ldS;
  bs.causal = kCausalSkipUpper;
  check_gemm(gemm_tf32_batched(BH, s.T, s.T, s.hd, heads_view(q, false, s, s.ldq, s.H, 1),
                               heads_view(k, false, s, s.ldk, s.Hkv, G), S, ldS, bs, 256, d_err, stream),
             "attention S = QK^T");
  const long long rows = static_cast<long long>(BH) * s.T;
  softmax_rows_kernel<<<blocks_for(rows * 32), 256, 0, stream>>>(S, ldS, s.T, rows, s.scale, lse);
  check("attention softmax");
  // O = P V, the K loop stopping at each row block's diagonal
  GemmBatch bo;
  bo.c_zdiv = s.H;
  bo.c_sb = static_cast<long long>(s.T) * s.ldo;
  bo.c_sh = s.hd;
  bo.causal = kCausalKBelow;
  check_gemm(gemm_tf32_batched(BH, s.T, s.hd, s.T, scores_view(S, false, s, ldS),
                               heads_view(v, true, s, s.ldv, s.Hkv, G), o, s.ldo, bo, tile_for(s.hd), d_err,
                               stream),
             "attention O = PV");
}

void attention_backward_tc(const AttnShape& s, const float* q, const float* k, const float* v, const float* o,
                           const float* lse, const float* dout, long long lddo, float* dq, float* dk, float* dv,
                           float* delta, float* S, float* dP, float* tmp, cudaStream_t stream) {
  DeviceContext& ctx = device_context();
  const int G = s.H / s.Hkv;
  const int BH = s.B * s.H;
  const long long ldS = attention_scores_ld(s.T);
  const long long rows = static_cast<long long>(BH) * s.T;
  attention_delta(s, o, dout, lddo, delta, stream);
  // S = Q K^T and dP = dO V^T on the causal part
  GemmBatch bs;
  bs.c_zdiv = BH;
  bs.c_sh = static_cast<long long>(s.T) * ldS;
  bs.causal = kCausalSkipUpper;
  check_gemm(gemm_tf32_batched(BH, s.T, s.T, s.hd, heads_view(q, false, s, s.ldq, s.H, 1),
                               heads_view(k, false, s, s.ldk, s.Hkv, G), S, ldS, bs, 256, ctx.d_err, stream),
             "attention S = QK^T (backward)");
  check_gemm(gemm_tf32_batched(BH, s.T, s.T, s.hd, heads_view(dout, false, s, lddo, s.H, 1),
                               heads_view(v, false, s, s.ldv, s.Hkv, G), dP, ldS, bs, 256, ctx.d_err, stream),
             "attention dP = dO V^T");
  softmax_bwd_rows_kernel<<<blocks_for(rows * 32), 256, 0, stream>>>(S, dP, ldS, s.T, rows, s.scale, lse, delta);
  check("attention softmax backward");
  const int bn = tile_for(s.hd);
  // dV = P^T dO and dK = dS^T Q: M = keys, K = queries from the key block on
  GemmBatch bk;
  bk.causal = kCausalKAbove;
  float* dv_out = G == 1 ? dv : tmp;
  float* dk_out = G == 1 ? dk : tmp;
  bk.c_zdiv = s.H;
  bk.c_sh = s.hd;
  const long long ld_kv = G == 1 ? s.ldk : static_cast<long long>(s.H) * s.hd;
  bk.c_sb = static_cast<long long>(s.T) * ld_kv;
  const long long tokens = static_cast<long long>(s.B) * s.T;
  check_gemm(gemm_tf32_batched(BH, s.T, s.hd, s.T, scores_view(S, true, s, ldS),
                               heads_view(dout, true, s, lddo, s.H, 1), dv_out, ld_kv, bk, bn, ctx.d_err, stream),
             "attention dV = P^T dO");
  if (G > 1) {
    group_sum_kernel<<<blocks_for(tokens * s.Hkv * s.hd), 256, 0, stream>>>(tmp, dv, tokens, s.Hkv, G, s.hd);
    check("attention dV group sum");
  }
  check_gemm(gemm_tf32_batched(BH, s.T, s.hd, s.T, scores_view(dP, true, s, ldS),
                               heads_view(q, true, s, s.ldq, s.H, 1), dk_out, ld_kv, bk, bn, ctx.d_err, stream),
             "attention dK = dS^T Q");
  if (G > 1) {
    group_sum_kernel<<<blocks_for(tokens * s.Hkv * s.hd), 256, 0, stream>>>(tmp, dk, tokens, s.Hkv, G, s.hd);
    check("attention dK group sum");
  }
  // dQ = dS K, the K loop stopping at the diagonal block
  GemmBatch bq;
  bq.c_zdiv = s.H;
  bq.c_sb = static_cast<long long>(s.T) * s.ldq;
  bq.c_sh = s.hd;
  bq.causal = kCausalKBelow;
  check_gemm(gemm_tf32_batched(BH, s.T, s.hd, s.T, scores_view(dP, false, s, ldS),
                               heads_view(k, true, s, s.ldk, s.Hkv, G), dq, s.ldq, bq, bn, ctx.d_err, stream),
             "attention dQ = dS K");
}

}  // namespace mm
