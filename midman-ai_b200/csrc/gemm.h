// Host interface of the tcgen05 TF32 GEMM (gemm.cu).
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

namespace mm {

// One GEMM operand. K-major: element (i, k) at ptr[i * ld + k]. MN-major:
// element (i, k) at ptr[k * ld + i]. ld is in elements and must be a multiple
// of 4; ptr must be 16-byte aligned (TMA requirements).
struct GemmOperand {
  const float* ptr;
  long long ld;
  bool mn_major;
};

enum GemmStatus : int {
  kGemmBadArgument = -101,
  kGemmMisaligned = -102,
  kGemmTensorMap = -103,
  kGemmLaunch = -104,
};

// Batched products (grid.z = batch). Batch z reads operand X at head
// (z % X.zdiv) / X.zgroup and batch z / X.zdiv of its 4-D view (the zdiv and
// zgroup of each BatchedOperand), and writes C at
// C + (z / c_zdiv) * c_sb + ((z % c_zdiv) / c_zgroup) * c_sh.
enum GemmCausal : int {
  kCausalNone = 0,
  kCausalSkipUpper = 1,  // output tiles entirely above the diagonal (n0 > m0 + 127) are not computed
  kCausalKBelow = 2,     // the K loop stops at m0 + 128 (keys up to the row block's last query)
  kCausalKAbove = 3,     // the K loop starts at m0 (queries from the key block's first key on)
};
struct GemmBatch {
  int a_zdiv = 1, a_zgroup = 1, b_zdiv = 1, b_zgroup = 1;
  long long c_sb = 0, c_sh = 0;
  int c_zdiv = 1, c_zgroup = 1;
  int causal = kCausalNone;
  // The K index of the operands' first column (a multiple of 32): a product over
  // one chunk of a longer K range applies the causal K bounds at their place in
  // the whole range (keys up to m0 + 127 - k_off, queries from m0 - k_off).
  int k_off = 0;
  int skip_empty = 0;  // set when R is C: tiles with an empty K range are left alone
};
// 4-D view of an operand, extents and strides in elements: `inner` contiguous
// (K for a K-major operand, M or N for an MN-major one), `rows` the other
// matrix dimension; heads and batches select the matrix.
struct BatchedOperand {
  const float* ptr;
  bool mn_major;
  long long inner, heads, rows, batches;
  long long head_stride, row_stride, batch_stride;
  int zdiv, zgroup;
};

// C[m, n] = sum_k A(m, k) B(n, k) (+ R[m, n] if R is not null; R may equal C).
// Asynchronous on `stream`; a pipeline timeout is reported through d_err.
int gemm_tf32(int M, int N, int K, GemmOperand A, GemmOperand B, float* C, long long ldc,
              const float* R, long long ldr, int* d_err, cudaStream_t stream);

// One term of a summed product: K columns of A times K columns of B.
struct GemmSegment {
  GemmOperand a, b;
  int K;
};
// C[m, n] = sum over the segments of sum_k A_s(m, k) B_s(n, k) (+ R[m, n]; R may
// equal C). Up to three segments with the same operand majors are summed in one
// accumulator by a single launch (their K steps one after another) when the
// shape runs on CTA pairs; otherwise one launch per segment accumulates into C.
int gemm_tf32_sum(int M, int N, const GemmSegment* segs, int nseg, float* C, long long ldc, const float* R,
                  long long ldr, int* d_err, cudaStream_t stream);

const char* gemm_status_string(int status);

// Kernels the GEMM functions have launched from the calling thread so far.
uint64_t gemm_launch_count();

// Streaming multiprocessors of the current device.
int sm_count();

// Two ticket words for persistent CTA-pair kernels launched on `stream` of
// device `dev`, shared by every such launch on the stream: each launch leaves
// them at zero. Null when the device's table of streams is full.
unsigned int* pair_ticket_counter(int dev, cudaStream_t stream);

// The batched form; bn (64, 128 or 256) is the output tile width. R (may be C)
// has C's layout and batch offsets and is added to each output element; an
// output tile whose causal K range is empty gets R alone (or zeros without R).
int gemm_tf32_batched(int batch, int M, int N, int K, const BatchedOperand& A, const BatchedOperand& B, float* C,
                      long long ldc, const GemmBatch& bt, int bn, int* d_err, cudaStream_t stream,
                      const float* R = nullptr);

// The batched form in 3xTF32 on split operands (hi/lo views of the same shape):
// C = Al Bh + Ah Bl + Ah Bh (+ R) in one launch, the tensor-memory accumulation
// restarted every 64 of K and the partial sums added in f32 in registers.
int gemm_3xtf32_batched(int batch, int M, int N, int K, const BatchedOperand& Ah, const BatchedOperand& Al,
                        const BatchedOperand& Bh, const BatchedOperand& Bl, float* C, long long ldc,
                        const GemmBatch& bt, int bn, int* d_err, cudaStream_t stream, const float* R = nullptr);

}  // namespace mm

namespace mm {
// hi = x rounded to TF32 (nearest), lo = (x - hi) rounded to TF32, for n values.
void split_tf32(const float* x, float* hi, float* lo, long long n, cudaStream_t stream);
// lo = (x - x with its low 13 mantissa bits cleared) rounded to TF32, for n
// values: the tensor core reads x itself as the hi part.
void split_lo_tf32(const float* x, float* lo, long long n, cudaStream_t stream);
// Same contract as gemm_tf32, computed as hi*hi + hi*lo + lo*hi (3xTF32).
// Uses the device scratch arena for the split operands.
int gemm_3xtf32(int M, int N, int K, GemmOperand A, GemmOperand B, float* C, long long ldc,
                const float* R, long long ldr, int* d_err, cudaStream_t stream);
// Lo copies of 3xTF32 operands kept between products on one stream, so that an
// operand used by consecutive products (a layer's input for its q, k and v
// projections; dY for dX and dW) is copied once. Entries hold the operand's
// address and extent, not its contents: a caller passes keep = true only when
// no kernel has written any operand of the products since the last call
// without it, which clears the cache. Operands above kMaxFloats are not kept.
struct X3LoCache {
  static constexpr int kSlots = 8;
  static constexpr long long kMaxFloats = 128ll << 20;
  struct Slot {
    const float* src = nullptr;
    long long n = 0, cap = 0;
    float* lo = nullptr;
    uint64_t stamp = 0;
  };
  Slot slot[kSlots];
  uint64_t clock = 0;
  X3LoCache() = default;
  X3LoCache(const X3LoCache&) = delete;
  X3LoCache& operator=(const X3LoCache&) = delete;
  ~X3LoCache();
};

// Same contract as gemm_tf32_sum in 3xTF32: one launch for up to three segments
// with the same majors when the shape runs on CTA pairs (the lo copies taken
// from, and kept in, `cache` when one is given).
int gemm_3xtf32_sum(int M, int N, const GemmSegment* segs, int nseg, float* C, long long ldc, const float* R,
                    long long ldr, int* d_err, cudaStream_t stream, X3LoCache* cache = nullptr, bool keep = false);
// The 3xTF32 CTA-pair kernel on split operands: hi[g] = (Ah, Bh, K), lo[g] =
// (Al, Bl, K) with the leading dimensions and majors of hi[g]; 1 to 3 segments
// with the same majors. C = sum_g (Al Bh + Ah Bl + Ah Bh) (+ R).
int gemm_3xtf32_pair_sum(int M, int N, const GemmSegment* hi, const GemmSegment* lo, int nseg, float* C,
                         long long ldc, const float* R, long long ldr, int* d_err, cudaStream_t stream);
// The exact-mode attention backward's score tiles in one launch: for every
// causal 128 x 128 tile (queries x keys) of every one of `batch` matrices,
// S = Q K^T and dP = dO V^T (3xTF32, K = hd; hi/lo views as gemm_3xtf32_batched,
// all K-major, dO addressed like Q and V like K), then P = exp(S * scale - lse)
// and dS = P (dP - delta) * scale (zero above the diagonal) as TF32 pairs: P to
// (Ph, Pl), dS to (Dh, Dl), [batch, T, ldS] through bt's output offsets; lse and
// delta are [batch * T]. Tiles wholly above the diagonal are not written.
int attention_scores_grad_3x(int batch, int T, int hd, const BatchedOperand& Qh, const BatchedOperand& Ql,
                             const BatchedOperand& Kh, const BatchedOperand& Kl, const BatchedOperand& Gh,
                             const BatchedOperand& Gl, const BatchedOperand& Vh, const BatchedOperand& Vl, float* Ph,
                             float* Pl, float* Dh, float* Dl, long long ldS, const GemmBatch& bt, const float* lse,
                             const float* delta, float scale, int* d_err, cudaStream_t stream);
// Whether products of this shape (n_k K steps of 32 in all) run on CTA pairs.
bool gemm_3xtf32_pair_suits(int M, int N, int n_k);
}  // namespace mm
