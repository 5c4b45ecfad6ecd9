// Per-device state shared by every kernel launcher: the device error flag the
// kernels' bounded waits write into, and a grow-only scratch arena.
#pragma once
#include <cuda_runtime.h>

#include <cstddef>
#include <string>

namespace mm {

struct DeviceContext {
  int device = -1;
  int* d_err = nullptr;        // kernel error flag (DeviceError codes), 0 = fine
  void* scratch = nullptr;     // grow-only arena for library-internal temporaries
  size_t scratch_bytes = 0;
  int sm_count = 0;
};

// The context of the current device, created on first use.
DeviceContext& device_context();

// Scratch of at least `bytes`, valid until the next call on this device. Work
// queued on other streams that still uses the old arena must be finished by the
// caller before growing it (the library only uses it on one stream at a time).
void* device_scratch(size_t bytes, cudaStream_t stream);

// Reads and clears the device error flag (synchronizes the stream).
int take_device_error(cudaStream_t stream);

std::string device_error_message(int code);

// Launches one thread that waits on a barrier nothing completes, bounded by
// timeout_ns: it records kErrWaitSelfTest in the error flag and returns.
void bounded_wait_selftest(unsigned long long timeout_ns, cudaStream_t stream);

// Message of the last failing kernel-level C ABI call on this thread
// (mm_gpu_last_error); the entry points of every capi_*.cu file set it.
void set_last_error(const std::string& msg);

// Throws std::runtime_error with the CUDA error text if `e` is not cudaSuccess.
void check_cuda(cudaError_t e, const char* what);

}  // namespace mm
