#include "device.h"

#include <mutex>
#include <stdexcept>
#include <vector>

#include "ptx.cuh"

namespace mm {

namespace {
std::mutex g_mu;
std::vector<DeviceContext> g_ctx;
}  // namespace

void check_cuda(cudaError_t e, const char* what) {
  if (e != cudaSuccess)
    throw std::runtime_error(std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")");
}

DeviceContext& device_context() {
  int dev = 0;
  check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_ctx.size() <= static_cast<size_t>(dev)) g_ctx.resize(dev + 1);
  DeviceContext& c = g_ctx[dev];
  if (c.device < 0) {
    c.device = dev;
    check_cuda(cudaMalloc(&c.d_err, 64), "cudaMalloc(error flag)");
    check_cuda(cudaMemset(c.d_err, 0, 64), "cudaMemset(error flag)");
    check_cuda(cudaDeviceGetAttribute(&c.sm_count, cudaDevAttrMultiProcessorCount, dev), "sm count");
  }
  return c;
}

void* device_scratch(size_t bytes, cudaStream_t stream) {
  DeviceContext& c = device_context();
  if (bytes > c.scratch_bytes) {
    if (c.scratch) {
      check_cuda(cudaStreamSynchronize(stream), "scratch sync");
      check_cuda(cudaFree(c.scratch), "cudaFree(scratch)");
      c.scratch = nullptr;
    }
    size_t want = bytes + bytes / 4 + (1u << 20);
    check_cuda(cudaMalloc(&c.scratch, want), "cudaMalloc(scratch)");
    c.scratch_bytes = want;
  }
  return c.scratch;
}

int take_device_error(cudaStream_t stream) {
  DeviceContext& c = device_context();
  int code = 0;
  check_cuda(cudaMemcpyAsync(&code, c.d_err, sizeof(int), cudaMemcpyDeviceToHost, stream), "read error flag");
  check_cuda(cudaStreamSynchronize(stream), "sync error flag");
  if (code) check_cuda(cudaMemsetAsync(c.d_err, 0, sizeof(int), stream), "clear error flag");
  return code;
}

namespace {
// One thread waits on a shared-memory barrier that nothing completes, through
// the same bounded wait the GEMM and attention pipelines use: after timeout_ns
// it records kErrWaitSelfTest in the error flag and the kernel returns. No copy
// or tensor-memory allocation is outstanding when it gives up.
__global__ void bounded_wait_selftest_kernel(int* err, unsigned long long timeout_ns) {
  __shared__ __align__(8) unsigned long long bar;
  const uint32_t a = smem_u32(&bar);
  mbar_init(a, 1);
  fence_barrier_init();
  mbar_wait(a, 0, err, kErrWaitSelfTest, timeout_ns);
}
}  // namespace

void bounded_wait_selftest(unsigned long long timeout_ns, cudaStream_t stream) {
  DeviceContext& c = device_context();
  bounded_wait_selftest_kernel<<<1, 1, 0, stream>>>(c.d_err, timeout_ns);
  check_cuda(cudaGetLastError(), "bounded wait self-test");
}

std::string device_error_message(int code) {
  switch (code) {
    case kErrNone: return "no device error";
    case kErrWaitFull: return "GEMM: UMMA issuer timed out waiting for a TMA stage";
    case kErrWaitEmpty: return "GEMM: TMA producer timed out waiting for a free stage";
    case kErrWaitAccum: return "GEMM: epilogue timed out waiting for the accumulator";
    case kErrWaitDrain: return "GEMM: teardown timed out draining TMA copies";
    case kErrBadShape: return "kernel rejected its shape";
    case kErrWaitUnit: return "GEMM: a role timed out waiting for its next work unit";
    case kErrIndex: return "a token id or target class is outside [0, vocab)";
    case kErrWaitSelfTest: return "self-test: a bounded wait ran out and the kernel returned";
    default: return "device error " + std::to_string(code);
  }
}

}  // namespace mm
