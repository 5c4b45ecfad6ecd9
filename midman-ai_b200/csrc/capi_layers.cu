// Kernel-level C ABI of the layers around the products (include/midman_gpu.h):
// RMSNorm, RoPE, SwiGLU, embedding, softmax cross-entropy, and the data-parallel
// gradient exchange. Each entry point checks its arguments on the host, then
// runs the same launcher the training step uses.
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstring>
#include <exception>
#include <string>
#include <thread>
#include <utility>
#include <vector>

#include "../../include/midman_gpu.h"
#include "device.h"
#include "kernels.h"
#include "nccl_api.h"

namespace {

thread_local std::string g_layer_error;

int32_t fail(int32_t code, const std::string& msg) {
  g_layer_error = msg;
  return code;
}

// Runs `body`; C++ exceptions become MM_GPU_ERR_DEVICE with their message.
// The message of a failing call is what mm_gpu_last_error returns next.
template <class F>
int32_t guarded(const char* what, F&& body) {
  int32_t rc;
  try {
    g_layer_error.clear();
    rc = body();
  } catch (const std::exception& e) {
    rc = fail(MM_GPU_ERR_DEVICE, std::string(what) + ": " + e.what());
  } catch (...) {
    rc = fail(MM_GPU_ERR_DEVICE, std::string(what) + ": unknown C++ exception");
  }
  mm::set_last_error(rc != MM_GPU_OK ? g_layer_error : std::string());
  return rc;
}

cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" {

int32_t mm_gpu_rmsnorm_forward(int32_t rows, int32_t dim, const float* x, const float* w, float eps, float* y,
                               float* rstd, void* stream) {
  return guarded("rmsnorm_forward", [&]() -> int32_t {
    if (rows < 0 || dim <= 0 || dim % 4 || dim > 8192)
      return fail(MM_GPU_ERR_SHAPE, "rmsnorm: dim must be a positive multiple of 4 up to 8192, rows >= 0");
    if (!(eps >= 0.0f) || !std::isfinite(eps)) return fail(MM_GPU_ERR_ARGUMENT, "rmsnorm: eps must be finite, >= 0");
    if (rows == 0) return MM_GPU_OK;
    if (!x || !w || !y || !rstd) return fail(MM_GPU_ERR_ARGUMENT, "rmsnorm: null pointer");
    if (!aligned16(x) || !aligned16(w) || !aligned16(y))
      return fail(MM_GPU_ERR_ARGUMENT, "rmsnorm: x, w and y must be 16-byte aligned");
    mm::rmsnorm_forward(x, w, rows, dim, eps, y, rstd, as_stream(stream));
    return MM_GPU_OK;
  });
}

int32_t mm_gpu_rmsnorm_backward(int32_t rows, int32_t dim, const float* x, const float* w, const float* rstd,
                                const float* dy, const float* dres, float* dx, float* dw, void* stream) {
  return guarded("rmsnorm_backward", [&]() -> int32_t {
    if (rows < 0 || dim <= 0 || dim % 4 || dim > 8192)
      return fail(MM_GPU_ERR_SHAPE, "rmsnorm: dim must be a positive multiple of 4 up to 8192, rows >= 0");
    if (!dw) return fail(MM_GPU_ERR_ARGUMENT, "rmsnorm: null pointer");
    cudaStream_t st = as_stream(stream);
    if (rows == 0) {
      mm::check_cuda(cudaMemsetAsync(dw, 0, static_cast<size_t>(dim) * sizeof(float), st), "dw");
      return MM_GPU_OK;
    }
    if (!x || !w || !rstd || !dy || !dx) return fail(MM_GPU_ERR_ARGUMENT, "rmsnorm: null pointer");
    if (!aligned16(x) || !aligned16(w) || !aligned16(dy) || !aligned16(dx) || (dres && !aligned16(dres)))
      return fail(MM_GPU_ERR_ARGUMENT, "rmsnorm: x, w, dy, dx and dres must be 16-byte aligned");
    const long long ws_floats = mm::rmsnorm_ws_floats(rows, dim);
    float* ws = static_cast<float*>(mm::device_scratch(static_cast<size_t>(ws_floats) * sizeof(float), st));
    mm::rmsnorm_backward(x, w, rstd, dy, rows, dim, dx, dres, dw, ws, st);
    return MM_GPU_OK;
  });
}

int32_t mm_gpu_rope(int32_t rows, int32_t seq, int32_t heads, int32_t head_dim, float* x, int64_t ld,
                    const float* cos_t, const float* sin_t, int32_t backward, void* stream) {
  return guarded("rope", [&]() -> int32_t {
    if (rows < 0 || seq <= 0 || heads <= 0 || head_dim <= 0 || (head_dim & 1) || rows % seq)
      return fail(MM_GPU_ERR_SHAPE, "rope: need rows = batch * seq, positive heads and an even head_dim");
    if (ld < static_cast<int64_t>(heads) * head_dim)
      return fail(MM_GPU_ERR_SHAPE, "rope: row stride smaller than the heads it holds");
    if (rows == 0) return MM_GPU_OK;
    if (!x || !cos_t || !sin_t) return fail(MM_GPU_ERR_ARGUMENT, "rope: null pointer");
    mm::rope(x, rows, seq, heads, head_dim, ld, cos_t, sin_t, backward != 0, as_stream(stream));
    return MM_GPU_OK;
  });
}

int32_t mm_gpu_swiglu_forward(int64_t n, const float* gate, const float* up, float* act, void* stream) {
  return guarded("swiglu_forward", [&]() -> int32_t {
    if (n < 0) return fail(MM_GPU_ERR_SHAPE, "swiglu: negative size");
    if (n == 0) return MM_GPU_OK;
    if (!gate || !up || !act) return fail(MM_GPU_ERR_ARGUMENT, "swiglu: null pointer");
    mm::swiglu_forward(gate, up, act, n, as_stream(stream));
    return MM_GPU_OK;
  });
}

int32_t mm_gpu_swiglu_backward(int64_t n, float* gate, float* up, const float* dact, void* stream) {
  return guarded("swiglu_backward", [&]() -> int32_t {
    if (n < 0) return fail(MM_GPU_ERR_SHAPE, "swiglu: negative size");
    if (n == 0) return MM_GPU_OK;
    if (!gate || !up || !dact) return fail(MM_GPU_ERR_ARGUMENT, "swiglu: null pointer");
    mm::swiglu_backward(gate, up, dact, n, as_stream(stream));
    return MM_GPU_OK;
  });
}

int32_t mm_gpu_embedding_forward(int32_t rows, const int32_t* ids, int32_t vocab, int32_t dim, const float* table,
                                 float* out, void* stream) {
  return guarded("embedding_forward", [&]() -> int32_t {
    if (rows < 0 || vocab <= 0 || dim <= 0 || dim % 4)
      return fail(MM_GPU_ERR_SHAPE, "embedding: need rows >= 0, vocab > 0 and dim a positive multiple of 4");
    if (rows == 0) return MM_GPU_OK;
    if (!ids || !table || !out) return fail(MM_GPU_ERR_ARGUMENT, "embedding: null pointer");
    if (!aligned16(table) || !aligned16(out))
      return fail(MM_GPU_ERR_ARGUMENT, "embedding: table and out must be 16-byte aligned");
    mm::embedding_forward(ids, rows, table, vocab, dim, out, mm::device_context().d_err, as_stream(stream));
    return MM_GPU_OK;
  });
}

int32_t mm_gpu_embedding_backward(int32_t rows, const int32_t* ids_host, int32_t vocab, int32_t dim,
                                  const float* dx, float* dtable, void* stream) {
  return guarded("embedding_backward", [&]() -> int32_t {
    if (rows < 0 || vocab <= 0 || dim <= 0)
      return fail(MM_GPU_ERR_SHAPE, "embedding: need rows >= 0, vocab > 0, dim > 0");
    if (rows == 0) return MM_GPU_OK;
    if (!ids_host || !dx || !dtable) return fail(MM_GPU_ERR_ARGUMENT, "embedding: null pointer");
    for (int32_t r = 0; r < rows; ++r)
      if (ids_host[r] < 0 || ids_host[r] >= vocab)
        return fail(MM_GPU_ERR_INDEX, "embedding: id " + std::to_string(ids_host[r]) + " at row " +
                                          std::to_string(r) + " is outside [0, " + std::to_string(vocab) + ")");
    // distinct ids with their rows in ascending order: each table row then adds
    // its rows' gradients in the order the reference's scatter-add visits them
    std::vector<std::pair<int32_t, int32_t>> order(rows);
    for (int32_t r = 0; r < rows; ++r) order[r] = {ids_host[r], r};
    std::sort(order.begin(), order.end());
    std::vector<int32_t> csr;  // [uniq (n_uniq) | offsets (n_uniq + 1) | rows (rows)]
    std::vector<int32_t> uniq, offs;
    for (int32_t i = 0; i < rows; ++i)
      if (i == 0 || order[i].first != order[i - 1].first) {
        uniq.push_back(order[i].first);
        offs.push_back(i);
      }
    offs.push_back(rows);
    const int n_uniq = static_cast<int>(uniq.size());
    csr.reserve(uniq.size() + offs.size() + rows);
    csr.insert(csr.end(), uniq.begin(), uniq.end());
    csr.insert(csr.end(), offs.begin(), offs.end());
    for (const auto& o : order) csr.push_back(o.second);
    cudaStream_t st = as_stream(stream);
    int32_t* d = static_cast<int32_t*>(mm::device_scratch(csr.size() * sizeof(int32_t), st));
    // a copy from pageable memory returns once the source has been read
    mm::check_cuda(cudaMemcpyAsync(d, csr.data(), csr.size() * sizeof(int32_t), cudaMemcpyHostToDevice, st),
                   "embedding index");
    mm::embedding_backward(d, d + n_uniq, d + 2 * n_uniq + 1, n_uniq, dx, dim, dtable, st);
    return MM_GPU_OK;
  });
}

int32_t mm_gpu_cross_entropy(int32_t rows, int32_t vocab, float* logits, int64_t ld, const int32_t* targets,
                             float grad_scale, float* row_loss, double* mean_loss, void* stream) {
  return guarded("cross_entropy", [&]() -> int32_t {
    if (rows <= 0 || vocab <= 0 || ld < vocab)
      return fail(MM_GPU_ERR_SHAPE, "cross_entropy: need rows > 0, vocab > 0 and ld >= vocab");
    if (!logits || !targets || !row_loss) return fail(MM_GPU_ERR_ARGUMENT, "cross_entropy: null pointer");
    if (!std::isfinite(grad_scale)) return fail(MM_GPU_ERR_ARGUMENT, "cross_entropy: grad_scale must be finite");
    cudaStream_t st = as_stream(stream);
    mm::cross_entropy(logits, ld, targets, rows, vocab, grad_scale, row_loss, mm::device_context().d_err, st);
    if (mean_loss) mm::mean_loss(row_loss, rows, mean_loss, st);
    return MM_GPU_OK;
  });
}

int32_t mm_gpu_wait_selftest(int32_t timeout_us, void* stream) {
  return guarded("wait_selftest", [&]() -> int32_t {
    if (timeout_us < 1 || timeout_us > 10000000)
      return fail(MM_GPU_ERR_ARGUMENT, "wait_selftest: timeout_us must lie in [1, 10000000]");
    mm::bounded_wait_selftest(static_cast<unsigned long long>(timeout_us) * 1000ull, as_stream(stream));
    return MM_GPU_OK;
  });
}

// ------------------------------------------------------------------ data-parallel exchange
//
// A communicator over the ranks of one data-parallel group, one per process
// and GPU, created from the 128-byte NCCL unique id rank 0 made
// (midman_nccl_unique_id) and shared out of band.
struct MmGpuComm {
  ncclComm_t comm = nullptr;
  int device = -1;
  int world = 0, rank = 0;
  bool aborted = false;
};

int32_t mm_gpu_comm_create(const uint8_t* nccl_id, int32_t world, int32_t rank, void** comm_out) {
  return guarded("comm_create", [&]() -> int32_t {
    if (!nccl_id || !comm_out) return fail(MM_GPU_ERR_ARGUMENT, "comm_create: null pointer");
    if (world < 1 || rank < 0 || rank >= world) return fail(MM_GPU_ERR_ARGUMENT, "comm_create: bad rank/world");
    *comm_out = nullptr;
    ncclUniqueId id;
    static_assert(sizeof(id) == 128, "NCCL unique id is 128 bytes");
    std::memcpy(&id, nccl_id, sizeof(id));
    auto* c = new MmGpuComm();
    c->world = world;
    c->rank = rank;
    mm::check_cuda(cudaGetDevice(&c->device), "cudaGetDevice");
    const ncclResult_t r = mm::nccl().CommInitRank(&c->comm, world, id, rank);
    if (r != ncclSuccess) {
      delete c;
      return fail(MM_GPU_ERR_DEVICE, std::string("ncclCommInitRank: ") + mm::nccl().GetErrorString(r));
    }
    *comm_out = c;
    return MM_GPU_OK;
  });
}

int32_t mm_gpu_comm_destroy(void* comm) {
  return guarded("comm_destroy", [&]() -> int32_t {
    auto* c = static_cast<MmGpuComm*>(comm);
    if (!c) return MM_GPU_OK;
    ncclResult_t r = ncclSuccess;
    if (c->comm) r = c->aborted ? ncclSuccess : mm::nccl().CommDestroy(c->comm);
    delete c;
    if (r != ncclSuccess) return fail(MM_GPU_ERR_DEVICE, std::string("ncclCommDestroy: ") + mm::nccl().GetErrorString(r));
    return MM_GPU_OK;
  });
}

int32_t mm_gpu_allreduce_bucket(void* comm, float* data, int64_t n, int32_t average, void* stream) {
  return guarded("allreduce_bucket", [&]() -> int32_t {
    auto* c = static_cast<MmGpuComm*>(comm);
    if (!c || !c->comm) return fail(MM_GPU_ERR_ARGUMENT, "allreduce_bucket: no communicator");
    if (c->aborted) return fail(MM_GPU_ERR_DEVICE, "allreduce_bucket: the communicator was aborted");
    if (n < 0) return fail(MM_GPU_ERR_SHAPE, "allreduce_bucket: negative size");
    if (n > 0 && !data) return fail(MM_GPU_ERR_ARGUMENT, "allreduce_bucket: null pointer");
    const ncclResult_t r = mm::nccl().AllReduce(data, data, static_cast<size_t>(n), ncclFloat,
                                                average ? ncclAvg : ncclSum, c->comm, as_stream(stream));
    if (r != ncclSuccess) return fail(MM_GPU_ERR_DEVICE, std::string("ncclAllReduce: ") + mm::nccl().GetErrorString(r));
    return MM_GPU_OK;
  });
}

int32_t mm_gpu_comm_wait(void* comm, void* stream, int32_t timeout_ms) {
  return guarded("comm_wait", [&]() -> int32_t {
    auto* c = static_cast<MmGpuComm*>(comm);
    if (!c || !c->comm) return fail(MM_GPU_ERR_ARGUMENT, "comm_wait: no communicator");
    if (c->aborted) return fail(MM_GPU_ERR_DEVICE, "comm_wait: the communicator was aborted");
    const cudaStream_t st = as_stream(stream);
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(std::max(timeout_ms, 0));
    for (;;) {
      const cudaError_t q = cudaStreamQuery(st);
      if (q == cudaSuccess) return MM_GPU_OK;
      if (q != cudaErrorNotReady) mm::check_cuda(q, "cudaStreamQuery");
      ncclResult_t async = ncclSuccess;
      const ncclResult_t r = mm::nccl().CommGetAsyncError(c->comm, &async);
      const bool failed = r != ncclSuccess || (async != ncclSuccess && async != ncclInProgress);
      if (failed || std::chrono::steady_clock::now() >= deadline) {
        // a peer is gone or the exchange hangs: abort so that the stream's
        // collectives end, then report (the communicator cannot be used again)
        mm::nccl().CommAbort(c->comm);
        c->aborted = true;
        return fail(MM_GPU_ERR_DEVICE, failed ? std::string("NCCL reported an asynchronous error: ") +
                                                    mm::nccl().GetErrorString(r != ncclSuccess ? r : async)
                                              : "comm_wait: the exchange did not finish within " +
                                                    std::to_string(timeout_ms) + " ms; communicator aborted");
      }
      std::this_thread::sleep_for(std::chrono::microseconds(200));
    }
  });
}

}  // extern "C"
