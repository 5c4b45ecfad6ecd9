// Kernel-level C ABI (include/midman_gpu.h): argument checks, then the launchers.
#include <cuda_runtime.h>

#include <cmath>
#include <exception>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/midman_gpu.h"
#include "attention.h"
#include "device.h"
#include "gemm.h"
#include "kernels.h"

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

void mm::set_last_error(const std::string& msg) { g_last_error = msg; }

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

int32_t mm_gpu_clip_adamw(int32_t n_tensors, const int64_t* numel, const int32_t* decay, float* p, const float* g,
                          float* m, float* v, double max_norm, double lr, double beta1, double beta2, double eps,
                          double weight_decay, uint64_t step, float* norm_out, void* stream) {
  return guarded([&]() -> int32_t {
    if (n_tensors < 0 || (n_tensors > 0 && (!numel || !decay || !p || !g || !m || !v)) || !norm_out)
      return fail(MM_GPU_ERR_ARGUMENT, "clip_adamw: null pointer or negative tensor count");
    if (step == 0) return fail(MM_GPU_ERR_ARGUMENT, "clip_adamw: step counts from 1");
    if (!(std::isfinite(lr) && lr >= 0.0) || !(std::isfinite(max_norm) && max_norm > 0.0))
      return fail(MM_GPU_ERR_ARGUMENT, "clip_adamw: lr and max_norm must be finite (max_norm positive)");
    // chunks of at most 16,384 elements inside one tensor, decay for the flagged ones
    std::vector<mm::AdamChunk> chunks;
    long long total = 0;
    for (int32_t i = 0; i < n_tensors; ++i) {
      if (numel[i] < 0) return fail(MM_GPU_ERR_ARGUMENT, "clip_adamw: negative tensor size");
      for (long long o = 0; o < numel[i]; o += 16384)
        chunks.push_back({total + o, static_cast<int>(numel[i] - o < 16384 ? numel[i] - o : 16384), decay[i] ? 1 : 0});
      total += numel[i];
    }
    // tensors start on 16-byte boundaries (the update reads four floats at a time)
    for (const mm::AdamChunk& c : chunks)
      if (c.offset % 4)
        return fail(MM_GPU_ERR_ARGUMENT, "clip_adamw: every tensor but the last must hold a multiple of 4 values");
    const cudaStream_t st = as_stream(stream);
    const size_t chunk_bytes = chunks.size() * sizeof(mm::AdamChunk);
    const size_t part_bytes = mm::kNormBlocks * sizeof(double);
    uint8_t* ws = static_cast<uint8_t*>(mm::device_scratch(part_bytes + 256 + chunk_bytes, st));
    double* partials = reinterpret_cast<double*>(ws);
    float* d_norm = reinterpret_cast<float*>(ws + part_bytes);
    mm::AdamChunk* d_chunks = reinterpret_cast<mm::AdamChunk*>(ws + part_bytes + 256);
    if (!chunks.empty())
      mm::check_cuda(cudaMemcpyAsync(d_chunks, chunks.data(), chunk_bytes, cudaMemcpyHostToDevice, st), "chunks");
    // clip.rs:29-59 (f64 sum of squares, scale by max/(norm+1e-6) above max) and
    // adamw.rs:141-217 (bias corrections in f64 for this step; nothing changes
    // when the norm is not finite)
    mm::sumsq_partials(g, total, partials, st);
    mm::finish_norm(partials, nullptr, static_cast<float>(max_norm), d_norm, st);
    const double t = static_cast<double>(step);
    const float bias1 = static_cast<float>(1.0 - std::pow(beta1, t));
    const float bias2_sqrt = static_cast<float>(std::sqrt(1.0 - std::pow(beta2, t)));
    const float flr = static_cast<float>(lr);
    mm::adamw_step(d_chunks, static_cast<int>(chunks.size()), p, g, m, v, 0, d_norm, flr, static_cast<float>(beta1),
                   static_cast<float>(beta2), static_cast<float>(eps), static_cast<float>(weight_decay), flr / bias1,
                   bias2_sqrt, st);
    mm::check_cuda(cudaMemcpyAsync(norm_out, d_norm, 3 * sizeof(float), cudaMemcpyDeviceToHost, st), "norm");
    mm::check_cuda(cudaStreamSynchronize(st), "clip_adamw");
    return MM_GPU_OK;
  });
}

int32_t mm_gpu_gemm_sum(int32_t m, int32_t n, int32_t nseg, const float* const* a, const int64_t* lda,
                        int32_t a_mn_major, const float* const* b, const int64_t* ldb, int32_t b_mn_major,
                        const int32_t* k, float* c, int64_t ldc, const float* r, int64_t ldr, void* stream) {
  return guarded([&]() -> int32_t {
    if (nseg < 1 || nseg > 8 || !a || !lda || !b || !ldb || !k)
      return fail(MM_GPU_ERR_ARGUMENT, "gemm_sum: 1 to 8 segments with their operands and sizes");
    mm::GemmSegment segs[8];
    for (int g = 0; g < nseg; ++g)
      segs[g] = mm::GemmSegment{{a[g], lda[g], a_mn_major != 0}, {b[g], ldb[g], b_mn_major != 0}, k[g]};
    mm::DeviceContext& ctx = mm::device_context();
    const int rc = mm::gemm_tf32_sum(m, n, segs, nseg, c, ldc, r, ldr, ctx.d_err, as_stream(stream));
    if (rc) return fail(rc == mm::kGemmLaunch ? MM_GPU_ERR_DEVICE : MM_GPU_ERR_ARGUMENT, mm::gemm_status_string(rc));
    return MM_GPU_OK;
  });
}

namespace {
int32_t attention_shape(int32_t B, int32_t T, int32_t H, int32_t Hkv, int32_t hd, int64_t ldq, int64_t ldk,
                        mm::AttnShape* s) {
  if (B <= 0 || T <= 0 || H <= 0 || Hkv <= 0 || hd <= 0 || H % Hkv != 0 || hd > 128 || (hd & 1))
    return fail(MM_GPU_ERR_SHAPE, "attention: need positive sizes, n_heads a multiple of n_kv_heads, even head_dim <= 128");
  if (ldq < static_cast<int64_t>(H) * hd || ldk < static_cast<int64_t>(Hkv) * hd)
    return fail(MM_GPU_ERR_SHAPE, "attention: row strides smaller than the heads they hold");
  *s = mm::AttnShape{B, T, H, Hkv, hd, ldq, ldk, ldk, ldq, 1.0f / std::sqrt(static_cast<float>(hd))};
  return MM_GPU_OK;
}
}  // namespace

int32_t mm_gpu_attention_forward(int32_t batch, int32_t seq, int32_t n_heads, int32_t n_kv_heads, int32_t head_dim,
                                 const float* q, const float* k, const float* v, int64_t ldq, int64_t ldk, float* o,
                                 float* lse, int32_t precision, void* stream) {
  return guarded([&]() -> int32_t {
    mm::AttnShape s;
    if (int32_t rc = attention_shape(batch, seq, n_heads, n_kv_heads, head_dim, ldq, ldk, &s)) return rc;
    if (!q || !k || !v || !o || !lse) return fail(MM_GPU_ERR_ARGUMENT, "attention: null pointer");
    cudaStream_t st = as_stream(stream);
    if (precision == MM_GPU_TF32 && mm::attention_flash_supported(s)) {
      mm::attention_forward_flash(s, q, k, v, o, lse, mm::device_context().d_err, st);
    } else if (precision == MM_GPU_3XTF32 && mm::attention_tc_supported(s)) {
      float* ws = static_cast<float*>(mm::device_scratch(
          static_cast<size_t>(mm::attention_3x_ws_floats(s, s.ldo)) * sizeof(float), st));
      mm::attention_forward_3x(s, q, k, v, o, lse, ws, mm::device_context().d_err, st);
    } else {
      mm::attention_forward(s, q, k, v, o, lse, st);
    }
    return MM_GPU_OK;
  });
}

int32_t mm_gpu_attention_backward(int32_t batch, int32_t seq, int32_t n_heads, int32_t n_kv_heads, int32_t head_dim,
                                  const float* q, const float* k, const float* v, const float* o, const float* lse,
                                  const float* dout, int64_t ldq, int64_t ldk, float* dq, float* dk, float* dv,
                                  int32_t precision, void* stream) {
  return guarded([&]() -> int32_t {
    mm::AttnShape s;
    if (int32_t rc = attention_shape(batch, seq, n_heads, n_kv_heads, head_dim, ldq, ldk, &s)) return rc;
    if (!q || !k || !v || !o || !lse || !dout || !dq || !dk || !dv)
      return fail(MM_GPU_ERR_ARGUMENT, "attention: null pointer");
    cudaStream_t st = as_stream(stream);
    const size_t rows = static_cast<size_t>(batch) * n_heads * seq;
    if (precision == MM_GPU_TF32 && mm::attention_flash_supported(s)) {
      float* delta = static_cast<float*>(mm::device_scratch(rows * sizeof(float), st));
      mm::attention_backward_flash(s, q, k, v, o, lse, dout, ldq, dq, dk, dv, delta, mm::device_context().d_err, st);
    } else if (precision == MM_GPU_3XTF32 && mm::attention_tc_supported(s)) {
      float* ws = static_cast<float*>(mm::device_scratch(
          static_cast<size_t>(mm::attention_3x_ws_floats(s, ldq)) * sizeof(float), st));
      mm::attention_backward_3x(s, q, k, v, o, lse, dout, ldq, dq, dk, dv, ws, mm::device_context().d_err, st);
    } else {
      float* delta = static_cast<float*>(mm::device_scratch(rows * sizeof(float), st));
      mm::attention_backward(s, q, k, v, o, lse, dout, ldq, dq, dk, dv, delta, st);
    }
    return MM_GPU_OK;
  });
}

}  // extern "C"

// ------------------------------------------------------------------ allocation-free attention forward
//
// Some callers cannot let this library call cudaMalloc: a process whose device
// memory is already fully reserved by its own pool (PyTorch's caching
// allocator, a serving engine's KV-cache arena) would see the library's
// allocation fail or push it out of memory, and cudaMalloc/cudaFree can
// synchronize the whole device, which a caller overlapping work on several
// streams cannot afford. mm_gpu_attention_forward's tensor-core path needs a
// score buffer, which it takes from a grow-only arena it allocates on demand;
// this variant takes it from a fixed array compiled into the library instead.
namespace {

// Score scratch of the allocation-free forward: batch * n_heads * seq * ld
// floats (ld = seq rounded up to a multiple of 4), at most 16 MiB. Every GPU
// that loads the library holds this array until the process exits. Every call
// shares it and it keeps the last call's contents; nothing in it has to start
// at zero, because each element a call reads was written earlier in the same
// call (score tiles above the diagonal are never read).
constexpr size_t kStaticScoreFloats = size_t(1) << 22;
static __device__ __align__(256) float g_static_scores[kStaticScoreFloats];

// Device address of g_static_scores per device. In host code the array's name
// is only a host-side stand-in, so the address is looked up once per device
// with that device current and kept for the life of the process: a
// cudaDeviceReset (which destroys the context holding the array) leaves the
// cached address stale, so the entry point must not be used after one.
std::mutex g_static_mu;
std::vector<float*> g_static_ptr;

float* static_scores(int device) {
  std::lock_guard<std::mutex> lock(g_static_mu);
  if (g_static_ptr.size() <= static_cast<size_t>(device)) g_static_ptr.resize(device + 1, nullptr);
  if (!g_static_ptr[device]) {
    float* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(reinterpret_cast<void**>(&p), g_static_scores);
    if (e != cudaSuccess) throw std::runtime_error(std::string("cudaGetSymbolAddress(score scratch): ") +
                                                   cudaGetErrorString(e));
    g_static_ptr[device] = p;
  }
  return g_static_ptr[device];
}

}  // namespace

extern "C" int32_t mm_gpu_attention_forward_noalloc(int32_t batch, int32_t seq, int32_t n_heads, int32_t n_kv_heads,
                                                    int32_t head_dim, const float* q, const float* k, const float* v,
                                                    int64_t ldq, int64_t ldk, float* o, float* lse,
                                                    int32_t* device_status, void* stream) {
  return guarded([&]() -> int32_t {
    mm::AttnShape s;
    if (int32_t rc = attention_shape(batch, seq, n_heads, n_kv_heads, head_dim, ldq, ldk, &s)) return rc;
    if (!q || !k || !v || !o || !lse || !device_status)
      return fail(MM_GPU_ERR_ARGUMENT, "attention (no-alloc): null pointer");
    if (head_dim != 32 && head_dim != 64 && head_dim != 128)
      return fail(MM_GPU_ERR_SHAPE, "attention (no-alloc): head_dim must be 32, 64 or 128");
    if (ldq % 4 || ldk % 4)
      return fail(MM_GPU_ERR_SHAPE, "attention (no-alloc): row strides ldq and ldk must be multiples of 4");
    // checked before anything is queued, so a refused call leaves o and lse alone
    for (const void* p : {static_cast<const void*>(q), static_cast<const void*>(k), static_cast<const void*>(v),
                          static_cast<const void*>(o)})
      if (reinterpret_cast<uintptr_t>(p) & 15u)
        return fail(MM_GPU_ERR_ARGUMENT, "attention (no-alloc): q, k, v and o must be 16-byte aligned");
    if (!mm::attention_tc_supported(s))
      return fail(MM_GPU_ERR_SHAPE, "attention (no-alloc): shape not supported by the tensor-core path");
    const size_t need = static_cast<size_t>(batch) * n_heads * seq * mm::attention_scores_ld(seq);
    if (need > kStaticScoreFloats)
      return fail(MM_GPU_ERR_SHAPE, "attention (no-alloc): batch * n_heads * seq * round4(seq) = " +
                                        std::to_string(need) + " floats exceeds the fixed score scratch of " +
                                        std::to_string(kStaticScoreFloats) + " floats (16 MiB)");
    int device = 0;
    const cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess) return fail(MM_GPU_ERR_DEVICE, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
    mm::attention_forward_tc(s, q, k, v, o, lse, static_scores(device), device_status, as_stream(stream));
    return MM_GPU_OK;
  });
}
