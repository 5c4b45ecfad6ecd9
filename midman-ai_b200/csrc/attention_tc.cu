// Causal grouped-query attention forward on the TF32 tensor cores through a
// score buffer: the score and probability matrices of every (batch, head) are
// formed by the batched tcgen05 GEMM (gemm.cu) restricted to the causal part,
// with the softmax as a row kernel between them. This is the path of the
// allocation-free entry point (a caller-given score buffer); training uses the
// fused flash kernels (flash_tc.cu, flash_bwd.cu), which keep the scores on chip.
//
// Forward (attention.rs:79-102):  S = Q K^T  ->  P = softmax(S * scale + mask), lse  ->  O = P V
// S/P live in a [B*H, T, ldS] buffer. Only the lower-triangular part is
// computed: output tiles above the diagonal are skipped and the K loop of O = P V
// stops at the diagonal block, so for causal T x T products about half the work
// of the dense product is done. Entries of a row past the query position but
// inside its 128-wide block are written as exact zeros, which is what a product
// whose K loop runs to the end of that block reads. K and V are addressed per
// key/value head (no copies for grouped-query sharing).
#include <cuda_runtime.h>

#include <cmath>
#include <stdexcept>
#include <string>

#include "attention.h"
#include "device.h"
#include "gemm.h"
#include "ptx.cuh"

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

// Round to the nearest TF32 value (ties away from zero), as split_tf32 does.
__device__ __forceinline__ float rn_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// The exact mode's softmax rows: as softmax_rows_kernel, but P goes out as its
// TF32 pair (hi = rn_tf32(p), lo = rn_tf32(p - hi)) for the three-term
// products, only up to the row's block end (the products read no further).
__global__ void softmax_split_rows_kernel(const float* __restrict__ S, float* __restrict__ Ph, float* __restrict__ Pl,
                                          long long ldS, int T, long long rows, float scale, float* __restrict__ lse) {
  const long long r = (blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x) / 32;
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  const int i = static_cast<int>(r % T);
  const float* row = S + r * ldS;
  float* hrow = Ph + r * ldS;
  float* lrow = Pl + r * ldS;
  const int n = i + 1, end = row_end(i, T);
  // exp(x) as 2^(x log2 e) on the special-function unit (relative error ~2^-22,
  // the TF32 pair's own level), with the scale folded into one multiply-add
  constexpr float kLog2e = 1.4426950408889634f;
  const float scale2 = scale * kLog2e;
  float m = -INFINITY;
  for (int j = lane; j < n; j += 32) m = fmaxf(m, row[j] * scale2);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  float s = 0.0f;
  for (int j = lane; j < n; j += 32) s += ex2_approx(fmaf(row[j], scale2, -m));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float inv = 1.0f / s;
  for (int j = lane; j < end; j += 32) {
    const float p = j < n ? ex2_approx(fmaf(row[j], scale2, -m)) * inv : 0.0f;
    const float h = rn_tf32(p);
    hrow[j] = h;
    lrow[j] = rn_tf32(p - h);
  }
  if (lse && lane == 0) lse[r] = (m + log2f(s)) / kLog2e;  // ln(sum exp): back from base 2
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

// ---------------------------------------------------------------- 3xTF32 products
// A TF32 number pair (hi, lo) per operand element, and a product formed as
// lo*hi + hi*lo + hi*hi in one launch of the batched 3xTF32 GEMM, which
// restarts its tensor-memory accumulation every 64 of K and adds the partial
// sums in f32, so the tensor core's accumulation error does not grow with the
// contraction's length; with `accumulate` the product is added to C.
struct Pair3 {
  BatchedOperand hi, lo;
};

void product3(int batch, int M, int N, int K, const Pair3& A, const Pair3& B, float* C, long long ldc,
              const GemmBatch& bt, int bn, bool accumulate, int* d_err, cudaStream_t stream, const char* what) {
  check_gemm(gemm_3xtf32_batched(batch, M, N, K, A.hi, A.lo, B.hi, B.lo, C, ldc, bt, bn, d_err, stream,
                                 accumulate ? C : nullptr),
             what);
}

// Head g of every key/value group of a token-major [B, T, H, hd] operand, as a
// batch over (b, kv head): z = b * Hkv + hk reads head hk * G + g.
BatchedOperand group_head_view(const float* p, bool mn, const AttnShape& s, long long ld, int g) {
  const int G = s.H / s.Hkv;
  return BatchedOperand{p + static_cast<long long>(g) * s.hd, mn, s.hd, s.Hkv, s.T, s.B,
                        static_cast<long long>(G) * s.hd, ld, static_cast<long long>(s.T) * ld, s.Hkv, 1};
}

// The same for the [B*H, T, ldS] score matrices, read with the keys as M
// (MN-major: A(key, query) = P[query][key]).
BatchedOperand group_scores_view(const float* p, const AttnShape& s, long long ldS, int g) {
  const int G = s.H / s.Hkv;
  const long long mat = static_cast<long long>(s.T) * ldS;
  return BatchedOperand{p + g * mat, true, s.T, s.Hkv, s.T, s.B, G * mat, ldS, static_cast<long long>(s.H) * mat,
                        s.Hkv, 1};
}

// The exact mode's workspace. The hi part of q, k, v and dO is the tensor
// itself (the tensor core reads its TF32 bits); only the lo parts are copies.
struct Ws3 {
  float *S, *D, *Xh, *Xl, *ql, *kl, *vl, *gl, *delta;
  const float *qh, *kh, *vh, *gh;
};

long long rows_footprint(const AttnShape& s, long long ld, int heads) {
  return (static_cast<long long>(s.B) * s.T - 1) * ld + static_cast<long long>(heads) * s.hd;
}

long long r4(long long n) { return (n + 63) & ~63ll; }

// Sizes (floats) of the pieces of the workspace, in carve's order.
struct Ws3Sizes {
  long long mat, nq, nk, nv, ng, nr;
  long long total() const { return 4 * mat + nq + nk + nv + ng + nr; }
};

Ws3Sizes ws3_sizes(const AttnShape& s, long long ld_dout) {
  return Ws3Sizes{r4(static_cast<long long>(s.B) * s.H * s.T * attention_scores_ld(s.T)),
                  r4(rows_footprint(s, s.ldq, s.H)),
                  r4(rows_footprint(s, s.ldk, s.Hkv)),
                  r4(rows_footprint(s, s.ldv, s.Hkv)),
                  r4(rows_footprint(s, ld_dout, s.H)),
                  r4(static_cast<long long>(s.B) * s.H * s.T)};
}

Ws3 carve(const AttnShape& s, float* ws, long long ld_dout, const float* q, const float* k, const float* v,
          const float* dout) {
  const Ws3Sizes z = ws3_sizes(s, ld_dout);
  const long long mat = z.mat, nq = z.nq, nk = z.nk, nv = z.nv, ng = z.ng, nr = z.nr;
  Ws3 w;
  float* p = ws;
  auto take = [&](long long n) { float* q = p; p += n; return q; };
  w.S = take(mat);
  w.D = take(mat);
  w.Xh = take(mat);
  w.Xl = take(mat);
  w.ql = take(nq);
  w.kl = take(nk);
  w.vl = take(nv);
  w.gl = take(ng);
  w.qh = q;
  w.kh = k;
  w.vh = v;
  w.gh = dout;
  w.delta = take(nr);
  return w;
}

// S = Q K^T (three terms), tiles above the diagonal skipped.
void scores3(const AttnShape& s, const Ws3& w, int* d_err, cudaStream_t st) {
  const int G = s.H / s.Hkv, BH = s.B * s.H;
  const long long ldS = attention_scores_ld(s.T);
  GemmBatch bs;
  bs.c_zdiv = BH;
  bs.c_sh = static_cast<long long>(s.T) * ldS;
  bs.causal = kCausalSkipUpper;
  product3(BH, s.T, s.T, s.hd, {heads_view(w.qh, false, s, s.ldq, s.H, 1), heads_view(w.ql, false, s, s.ldq, s.H, 1)},
           {heads_view(w.kh, false, s, s.ldk, s.Hkv, G), heads_view(w.kl, false, s, s.ldk, s.Hkv, G)}, w.S, ldS, bs,
           128, false, d_err, st, "attention (3xTF32) S = QK^T");
}

// P = softmax(S) of every score row into (Xh, Xl) as its TF32 pair (and lse).
void softmax_split(const AttnShape& s, const Ws3& w, float* lse, cudaStream_t st) {
  const long long rows = static_cast<long long>(s.B) * s.H * s.T;
  softmax_split_rows_kernel<<<blocks_for(rows * 32), 256, 0, st>>>(w.S, w.Xh, w.Xl, attention_scores_ld(s.T), s.T,
                                                                  rows, s.scale, lse);
  check("attention softmax");
}

}  // namespace

long long attention_3x_ws_floats(const AttnShape& s, long long ld_dout) { return ws3_sizes(s, ld_dout).total(); }

void attention_forward_3x(const AttnShape& s, const float* q, const float* k, const float* v, float* o, float* lse,
                          float* ws, int* d_err, cudaStream_t st) {
  const Ws3 w = carve(s, ws, s.ldo, q, k, v, nullptr);
  const int G = s.H / s.Hkv, BH = s.B * s.H;
  const long long ldS = attention_scores_ld(s.T);
  split_lo_tf32(q, w.ql, rows_footprint(s, s.ldq, s.H), st);
  split_lo_tf32(k, w.kl, rows_footprint(s, s.ldk, s.Hkv), st);
  split_lo_tf32(v, w.vl, rows_footprint(s, s.ldv, s.Hkv), st);
  scores3(s, w, d_err, st);
  softmax_split(s, w, lse, st);
  // O = P V, each row block's K loop ending at its diagonal
  GemmBatch bo;
  bo.c_zdiv = s.H;
  bo.c_sb = static_cast<long long>(s.T) * s.ldo;
  bo.c_sh = s.hd;
  bo.causal = kCausalKBelow;
  product3(BH, s.T, s.hd, s.T, {scores_view(w.Xh, false, s, ldS), scores_view(w.Xl, false, s, ldS)},
           {heads_view(w.vh, true, s, s.ldv, s.Hkv, G), heads_view(w.vl, true, s, s.ldv, s.Hkv, G)}, o, s.ldo, bo,
           tile_for(s.hd), false, d_err, st, "attention (3xTF32) O = PV");
}

void attention_backward_3x(const AttnShape& s, const float* q, const float* k, const float* v, const float* o,
                           const float* lse, const float* dout, long long lddo, float* dq, float* dk, float* dv,
                           float* ws, int* d_err, cudaStream_t st) {
  const Ws3 w = carve(s, ws, lddo, q, k, v, dout);
  const int G = s.H / s.Hkv, BH = s.B * s.H, BHkv = s.B * s.Hkv;
  const long long ldS = attention_scores_ld(s.T);
  split_lo_tf32(q, w.ql, rows_footprint(s, s.ldq, s.H), st);
  split_lo_tf32(k, w.kl, rows_footprint(s, s.ldk, s.Hkv), st);
  split_lo_tf32(v, w.vl, rows_footprint(s, s.ldv, s.Hkv), st);
  split_lo_tf32(dout, w.gl, rows_footprint(s, lddo, s.H), st);
  attention_delta(s, o, dout, lddo, w.delta, st);
  // One launch for the score tiles: S = QK^T and dP = dO V^T, then
  // P = exp(S * scale - lse) (the forward's lse) and dS = P (dP - delta) * scale,
  // as TF32 pairs: P into (Xh, Xl), dS into (S, D)
  {
    GemmBatch bs;
    bs.c_zdiv = BH;
    bs.c_sh = static_cast<long long>(s.T) * ldS;
    check_gemm(attention_scores_grad_3x(
                   BH, s.T, s.hd, heads_view(w.qh, false, s, s.ldq, s.H, 1), heads_view(w.ql, false, s, s.ldq, s.H, 1),
                   heads_view(w.kh, false, s, s.ldk, s.Hkv, G), heads_view(w.kl, false, s, s.ldk, s.Hkv, G),
                   heads_view(w.gh, false, s, lddo, s.H, 1), heads_view(w.gl, false, s, lddo, s.H, 1),
                   heads_view(w.vh, false, s, s.ldv, s.Hkv, G), heads_view(w.vl, false, s, s.ldv, s.Hkv, G), w.Xh,
                   w.Xl, w.S, w.D, ldS, bs, lse, w.delta, s.scale, d_err, st),
               "attention (3xTF32) P, dS");
  }
  // dV = P^T dO, summed over each key/value head's group; each key row block's
  // K loop starting at its first key
  GemmBatch bk;
  bk.c_zdiv = s.Hkv;
  bk.c_sb = static_cast<long long>(s.T) * s.ldv;
  bk.c_sh = s.hd;
  bk.causal = kCausalKAbove;
  for (int g = 0; g < G; ++g)
    product3(BHkv, s.T, s.hd, s.T, {group_scores_view(w.Xh, s, ldS, g), group_scores_view(w.Xl, s, ldS, g)},
             {group_head_view(w.gh, true, s, lddo, g), group_head_view(w.gl, true, s, lddo, g)}, dv, s.ldv, bk,
             tile_for(s.hd), g > 0, d_err, st, "attention (3xTF32) dV = P^T dO");
  // dK = dS^T Q, summed over the group
  bk.c_sb = static_cast<long long>(s.T) * s.ldk;
  for (int g = 0; g < G; ++g)
    product3(BHkv, s.T, s.hd, s.T, {group_scores_view(w.S, s, ldS, g), group_scores_view(w.D, s, ldS, g)},
             {group_head_view(w.qh, true, s, s.ldq, g), group_head_view(w.ql, true, s, s.ldq, g)}, dk, s.ldk, bk,
             tile_for(s.hd), g > 0, d_err, st, "attention (3xTF32) dK = dS^T Q");
  // dQ = dS K, K = keys ending at each row block's diagonal
  GemmBatch bq;
  bq.c_zdiv = s.H;
  bq.c_sb = static_cast<long long>(s.T) * s.ldq;
  bq.c_sh = s.hd;
  bq.causal = kCausalKBelow;
  product3(BH, s.T, s.hd, s.T, {scores_view(w.S, false, s, ldS), scores_view(w.D, false, s, ldS)},
           {heads_view(w.kh, true, s, s.ldk, s.Hkv, G), heads_view(w.kl, true, s, s.ldk, s.Hkv, G)}, dq, s.ldq, bq,
           tile_for(s.hd), false, d_err, st, "attention (3xTF32) dQ = dS K");
}

long long attention_scores_ld(int T) { return (T + 3) & ~3ll; }

bool attention_tc_supported(const AttnShape& s) {
  return (s.hd == 32 || s.hd == 64 || s.hd == 128) && s.H % s.Hkv == 0 && s.ldq % 4 == 0 && s.ldk % 4 == 0 &&
         s.ldv % 4 == 0 && s.ldo % 4 == 0;
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

}  // namespace mm
