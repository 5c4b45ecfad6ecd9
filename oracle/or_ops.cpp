// Oracle part 2: the three matrix-product kernels in the reference's loop order.
// Test infrastructure only (see oracle.h).
//
// crates/midman-tensor/src/kernels.rs:87-109: every C[i][j] adds its products
// in ascending order of the inner index, a separate multiply and add each
// (built with -ffp-contract=off). crates/midman-tensor/src/kernels_avx.rs:1-20
// gets the same bits faster by keeping a tile of C in registers for the whole
// inner loop (separate _mm256_mul_ps / _mm256_add_ps, never a fused
// multiply-add). The kernel below does the same: a tile of 4 rows x 16 columns
// accumulates A(i,p) * B[p][j] for p ascending from the current C value, so
// every element sees exactly the scalar loop's sequence of roundings. A strip
// of 16 columns of B is copied into a contiguous buffer once and then serves
// every row of C (the copy changes no arithmetic); rows of C are independent,
// so they may run on several threads without changing any element's result.
#include <immintrin.h>
#include <algorithm>
#include <omp.h>

#include <vector>

#include "oracle_internal.h"

namespace orc {

void set_threads(int n) {
  if (n > 0) omp_set_num_threads(n);
}

namespace {

constexpr size_t kRows = 4;     // rows of C per register tile

// R rows x V vectors of 8 columns: C(i, j) += sum_p A(i, p) * B[p][j], p ascending.
// A(i, p) = a[i * rs + p * cs].
template <size_t R, size_t V>
inline void tile(const float* a, size_t rs, size_t cs, const float* b, size_t ldb, float* c, size_t ldc, size_t k) {
  __m256 acc[R][V];
  for (size_t r = 0; r < R; ++r)
    for (size_t v = 0; v < V; ++v) acc[r][v] = _mm256_loadu_ps(c + r * ldc + 8 * v);
  for (size_t p = 0; p < k; ++p) {
    const float* bp = b + p * ldb;
    __m256 bv[V];
    for (size_t v = 0; v < V; ++v) bv[v] = _mm256_loadu_ps(bp + 8 * v);
    for (size_t r = 0; r < R; ++r) {
      const __m256 av = _mm256_set1_ps(a[r * rs + p * cs]);
      for (size_t v = 0; v < V; ++v) acc[r][v] = _mm256_add_ps(acc[r][v], _mm256_mul_ps(av, bv[v]));
    }
  }
  for (size_t r = 0; r < R; ++r)
    for (size_t v = 0; v < V; ++v) _mm256_storeu_ps(c + r * ldc + 8 * v, acc[r][v]);
}

// Fewer than 8 columns left: the scalar loop, p ascending per element.
template <size_t R>
inline void tail(const float* a, size_t rs, size_t cs, const float* b, size_t ldb, float* c, size_t ldc, size_t k,
                 size_t w) {
  for (size_t r = 0; r < R; ++r)
    for (size_t j = 0; j < w; ++j) {
      float acc = c[r * ldc + j];
      for (size_t p = 0; p < k; ++p) acc += a[r * rs + p * cs] * b[p * ldb + j];
      c[r * ldc + j] = acc;
    }
}

// Rows [i0, i1) of C over the columns [j, j + w) of one strip, B's strip already
// packed contiguously (row stride w), so that the inner loop reads it in order.
template <size_t V>
inline void strip(const float* a, size_t rs, size_t cs, const float* bp, float* c, size_t ldc, size_t k, size_t i0,
                  size_t i1) {
  size_t i = i0;
  for (; i + kRows <= i1; i += kRows) tile<kRows, V>(a + i * rs, rs, cs, bp, 8 * V, c + i * ldc, ldc, k);
  switch (i1 - i) {
    case 3: tile<3, V>(a + i * rs, rs, cs, bp, 8 * V, c + i * ldc, ldc, k); break;
    case 2: tile<2, V>(a + i * rs, rs, cs, bp, 8 * V, c + i * ldc, ldc, k); break;
    case 1: tile<1, V>(a + i * rs, rs, cs, bp, 8 * V, c + i * ldc, ldc, k); break;
    default: break;
  }
}

// Rows [i0, i1) of C, all columns: strip by strip of 16 (then 8, then the tail).
inline void rows_range(const float* a, size_t rs, size_t cs, const float* b, size_t ldb, float* c, size_t ldc,
                       size_t k, size_t n, size_t i0, size_t i1, std::vector<float>& pack) {
  if (i0 >= i1) return;
  std::vector<float> apack;
  if (cs != 1) {
    // A is read down its columns (A^T B): copy the band's rows into row-major
    // order first, so that the tile's broadcasts walk memory in order.
    apack.resize((i1 - i0) * k);
    for (size_t p = 0; p < k; ++p)
      for (size_t i = i0; i < i1; ++i) apack[(i - i0) * k + p] = a[i * rs + p * cs];
    a = apack.data() - i0 * k;
    rs = k;
    cs = 1;
  }
  pack.resize(k * 16);
  size_t j = 0;
  for (; j + 8 <= n; j += (n - j >= 16 ? 16 : 8)) {
    const size_t w = n - j >= 16 ? 16 : 8;
    for (size_t p = 0; p < k; ++p)
      for (size_t q = 0; q < w; ++q) pack[p * w + q] = b[p * ldb + j + q];
    if (w == 16)
      strip<2>(a, rs, cs, pack.data(), c + j, ldc, k, i0, i1);
    else
      strip<1>(a, rs, cs, pack.data(), c + j, ldc, k, i0, i1);
  }
  if (j < n)
    for (size_t i = i0; i < i1; ++i) tail<1>(a + i * rs, rs, cs, b + j, ldb, c + i * ldc + j, ldc, k, n - j);
}

}  // namespace

void gemm_strided_serial(const float* a, size_t rs, size_t cs, const float* b, size_t ldb, float* c, size_t ldc,
                         size_t m, size_t k, size_t n) {
  std::vector<float> pack;
  rows_range(a, rs, cs, b, ldb, c, ldc, k, n, 0, m, pack);
}

// C[m,n] += A(i,p) B[p][j] on all threads, each taking a band of rows.
static void gemm_strided(const float* a, size_t rs, size_t cs, const float* b, float* c, size_t m, size_t k,
                         size_t n) {
  if (m * k * n <= (1u << 16)) {
    gemm_strided_serial(a, rs, cs, b, n, c, n, m, k, n);
    return;
  }
  const long long blocks = static_cast<long long>((m + kRows - 1) / kRows);
#pragma omp parallel
  {
    const long long nt = omp_get_num_threads(), t = omp_get_thread_num();
    const size_t i0 = static_cast<size_t>(blocks * t / nt) * kRows;
    const size_t i1 = std::min(m, static_cast<size_t>(blocks * (t + 1) / nt) * kRows);
    std::vector<float> pack;
    rows_range(a, rs, cs, b, n, c, n, k, n, i0, i1, pack);
  }
}

// kernels.rs:90-98 scalar::gemm_nn
void gemm_nn(const float* a, const float* b, float* c, size_t m, size_t k, size_t n) {
  gemm_strided(a, k, 1, b, c, m, k, n);
}

// kernels.rs:66-75 gemm_nt: B [n, k] is copied into a [k, n] layout, then gemm_nn.
void gemm_nt(const float* a, const float* b, float* c, size_t m, size_t k, size_t n) {
  std::vector<float> bt(k * n);
#pragma omp parallel for schedule(static) if (k * n > (1u << 16))
  for (long long j = 0; j < static_cast<long long>(n); ++j)
    for (size_t p = 0; p < k; ++p) bt[p * n + j] = b[j * k + p];
  gemm_nn(a, bt.data(), c, m, k, n);
}

// kernels.rs:101-109 scalar::gemm_tn: C[i][j] += sum_p A[p][i] * B[p][j], p ascending.
void gemm_tn(const float* a, const float* b, float* c, size_t k, size_t m, size_t n) {
  gemm_strided(a, 1, m, b, c, m, k, n);
}

}  // namespace orc
