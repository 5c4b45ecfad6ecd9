// 3xTF32 ("exact") mode of the GEMM: each operand is split into a TF32-exact
// high part and the remainder, x = hi + lo with hi = x with its low 13 mantissa
// bits cleared, and the product is formed as hi*hi + hi*lo + lo*hi on the TF32
// tensor cores (the lo*lo term is below f32 resolution). This is the split of
// Ootomo & Yokota (2022); it recovers close to f32 accuracy at 3x the MMA work.
#include <cuda_runtime.h>

#include "device.h"
#include "gemm.h"

namespace mm {

namespace {

__global__ void split_tf32_kernel(const float* __restrict__ x, float* __restrict__ hi,
                                  float* __restrict__ lo, long long n) {
  long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (; i < n; i += stride) {
    const float v = x[i];
    const float h = __uint_as_float(__float_as_uint(v) & 0xFFFFE000u);
    hi[i] = h;
    lo[i] = v - h;  // exact in f32
  }
}

// Elements an operand of `rows` x `cols` with leading dimension `ld` spans.
long long footprint(long long rows, long long cols, long long ld) {
  return rows == 0 || cols == 0 ? 0 : (rows - 1) * ld + cols;
}

void split(const float* x, float* hi, float* lo, long long n, cudaStream_t s) {
  if (n <= 0) return;
  const int threads = 256;
  long long blocks = (n + threads - 1) / threads;
  if (blocks > 148 * 32) blocks = 148 * 32;
  split_tf32_kernel<<<static_cast<int>(blocks), threads, 0, s>>>(x, hi, lo, n);
}

long long round4(long long n) { return (n + 3) & ~3ll; }

}  // namespace

int gemm_3xtf32(int M, int N, int K, GemmOperand A, GemmOperand B, float* C, long long ldc,
                const float* R, long long ldr, int* d_err, cudaStream_t stream) {
  if (M == 0 || N == 0 || K == 0) return gemm_tf32(M, N, K, A, B, C, ldc, R, ldr, d_err, stream);
  const long long na = A.mn_major ? footprint(K, M, A.ld) : footprint(M, K, A.ld);
  const long long nb = B.mn_major ? footprint(K, N, B.ld) : footprint(N, K, B.ld);
  const long long pa = round4(na), pb = round4(nb);
  float* ws = static_cast<float*>(device_scratch(static_cast<size_t>(2 * pa + 2 * pb) * sizeof(float), stream));
  float *a_hi = ws, *a_lo = ws + pa, *b_hi = ws + 2 * pa, *b_lo = ws + 2 * pa + pb;
  split(A.ptr, a_hi, a_lo, na, stream);
  split(B.ptr, b_hi, b_lo, nb, stream);
  GemmOperand Ah{a_hi, A.ld, A.mn_major}, Al{a_lo, A.ld, A.mn_major};
  GemmOperand Bh{b_hi, B.ld, B.mn_major}, Bl{b_lo, B.ld, B.mn_major};
  // Small terms first, then the large one, so the small ones are not rounded
  // away against a large partial sum before they are combined (one accumulator
  // over the three K ranges when the shape runs on CTA pairs).
  const GemmSegment terms[3] = {{Al, Bh, K}, {Ah, Bl, K}, {Ah, Bh, K}};
  return gemm_tf32_sum(M, N, terms, 3, C, ldc, R, ldr, d_err, stream);
}

}  // namespace mm
