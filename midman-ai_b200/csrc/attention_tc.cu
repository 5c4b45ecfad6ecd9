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
