// Oracle part 2: the three matrix-product kernels in the reference's loop order.
// Test infrastructure only (see oracle.h).
//
// crates/midman-tensor/src/kernels.rs:87-109: every C[i][j] adds its products
// in ascending order of the inner index, a separate multiply and add each
// (built with -ffp-contract=off). Rows of C are independent, so they may run on
// several threads without changing any element's result.
#include <omp.h>

#include <vector>

#include "oracle_internal.h"

namespace orc {

void set_threads(int n) {
  if (n > 0) omp_set_num_threads(n);
}

// kernels.rs:90-98 scalar::gemm_nn
void gemm_nn(const float* a, const float* b, float* c, size_t m, size_t k, size_t n) {
#pragma omp parallel for schedule(static) if (m * k * n > (1u << 16))
  for (long long i = 0; i < static_cast<long long>(m); ++i) {
    const float* arow = a + i * k;
    float* crow = c + i * n;
    for (size_t p = 0; p < k; ++p) {
      const float aip = arow[p];
      const float* brow = b + p * n;
      for (size_t j = 0; j < n; ++j) crow[j] += aip * brow[j];
    }
  }
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
#pragma omp parallel for schedule(static) if (m * k * n > (1u << 16))
  for (long long i = 0; i < static_cast<long long>(m); ++i) {
    float* crow = c + i * n;
    for (size_t p = 0; p < k; ++p) {
      const float api = a[p * m + i];
      const float* brow = b + p * n;
      for (size_t j = 0; j < n; ++j) crow[j] += api * brow[j];
    }
  }
}

}  // namespace orc
