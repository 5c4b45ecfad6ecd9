// Host interface of the tcgen05 TF32 GEMM (gemm.cu).
#pragma once
#include <cuda_runtime.h>

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

// C[m, n] = sum_k A(m, k) B(n, k) (+ R[m, n] if R is not null; R may equal C).
// Asynchronous on `stream`; a pipeline timeout is reported through d_err.
int gemm_tf32(int M, int N, int K, GemmOperand A, GemmOperand B, float* C, long long ldc,
              const float* R, long long ldr, int* d_err, cudaStream_t stream);

const char* gemm_status_string(int status);

}  // namespace mm

namespace mm {
// Same contract as gemm_tf32, computed as hi*hi + hi*lo + lo*hi (3xTF32).
// Uses the device scratch arena for the split operands.
int gemm_3xtf32(int M, int N, int K, GemmOperand A, GemmOperand B, float* C, long long ldc,
                const float* R, long long ldr, int* d_err, cudaStream_t stream);
}  // namespace mm
