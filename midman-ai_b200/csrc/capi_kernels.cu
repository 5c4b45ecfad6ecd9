// Kernel-level C ABI (include/midman_gpu.h): argument checks, then the launchers.
#include <cuda_runtime.h>

#include <exception>
#include <string>

#include "../../include/midman_gpu.h"
#include "device.h"
#include "gemm.h"

namespace {
thread_local std::string g_last_error;

int32_t fail(int32_t code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

template <class F>
int32_t guarded(F&& body) {
  try {
    g_last_error.clear();
    return body();
  } catch (const std::exception& e) {
    return fail(MM_GPU_ERR_DEVICE, e.what());
  } catch (...) {
    return fail(MM_GPU_ERR_DEVICE, "unknown C++ exception");
  }
}

cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }
}  // namespace

extern "C" {

const char* mm_gpu_last_error(void) { return g_last_error.c_str(); }

int32_t mm_gpu_device_status(void* stream) {
  return guarded([&]() -> int32_t {
    const int code = mm::take_device_error(as_stream(stream));
    if (code) return fail(MM_GPU_ERR_DEVICE, mm::device_error_message(code));
    return MM_GPU_OK;
  });
}

int32_t mm_gpu_gemm(int32_t m, int32_t n, int32_t k, const float* a, int64_t lda, int32_t a_mn_major,
                    const float* b, int64_t ldb, int32_t b_mn_major, float* c, int64_t ldc,
                    const float* r, int64_t ldr, int32_t precision, void* stream) {
  return guarded([&]() -> int32_t {
    if (precision != MM_GPU_TF32 && precision != MM_GPU_3XTF32)
      return fail(MM_GPU_ERR_ARGUMENT, "precision must be MM_GPU_TF32 or MM_GPU_3XTF32");
    mm::DeviceContext& ctx = mm::device_context();
    mm::GemmOperand A{a, lda, a_mn_major != 0}, B{b, ldb, b_mn_major != 0};
    const int rc = precision == MM_GPU_TF32
                       ? mm::gemm_tf32(m, n, k, A, B, c, ldc, r, ldr, ctx.d_err, as_stream(stream))
                       : mm::gemm_3xtf32(m, n, k, A, B, c, ldc, r, ldr, ctx.d_err, as_stream(stream));
    if (rc) return fail(rc == mm::kGemmLaunch ? MM_GPU_ERR_DEVICE : MM_GPU_ERR_ARGUMENT, mm::gemm_status_string(rc));
    return MM_GPU_OK;
  });
}

}  // extern "C"
