// Device tensors with a recording autograd tape (include/midman_tensor.h).
//
// The reference's midman-tensor keeps a tensor's values in host memory and, when
// an operation has an input that tracks gradients, records a node holding the
// inputs and a backward closure (crates/midman-tensor/src/autograd.rs:27-41);
// Tensor::backward orders the reachable nodes depth first, seeds the output with
// 1 and runs the closures from the output toward the leaves, summing gradients
// that reach a tensor from several uses (autograd.rs:44-124). This file keeps the
// same rules with the values in HBM: each operation launches its kernels at once
// on the tape's stream, and the recorded backward launches the gradient kernels,
// accumulating into per-tensor gradient buffers on the device. Operations are the
// fused layer kernels of this library (a GEMM for matmul, one kernel for RMSNorm,
// RoPE, SwiGLU, causal attention, cross-entropy) rather than the reference's
// primitives, so a graph has a node per layer op instead of per arithmetic step.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <functional>
#include <map>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <tuple>
#include <unordered_map>
#include <unordered_set>
#include <utility>
#include <vector>

#include "../../include/midman_gpu.h"
#include "../../include/midman_tensor.h"
#include "attention.h"
#include "device.h"
#include "gemm.h"
#include "host.h"
#include "kernels.h"

namespace mm {
namespace {

// ---------------------------------------------------------------- small kernels
__global__ void mul_kernel(const float* __restrict__ a, const float* __restrict__ b, float* __restrict__ out,
                           long long n, int accumulate) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const float p = a[i] * b[i];
    out[i] = accumulate ? out[i] + p : p;
  }
}

// out += s[0] * x (s on the device: the upstream gradient of a scalar)
__global__ void axpy_dev_kernel(const float* __restrict__ s, const float* __restrict__ x, float* __restrict__ out,
                                long long n) {
  const float a = s[0];
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x)
    out[i] += a * x[i];
}

__global__ void fill_kernel(float* out, float v, long long n) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x)
    out[i] = v;
}

__global__ void double_to_float_kernel(const double* in, float* out) { out[0] = static_cast<float>(in[0]); }

int blocks_for(long long n) {
  long long b = (n + 255) / 256;
  return static_cast<int>(std::max(1ll, std::min(b, 148ll * 16)));
}

// ---------------------------------------------------------------- tensors and nodes
struct Storage {
  float* ptr = nullptr;
  size_t n = 0;
  cudaStream_t stream = nullptr;
  Storage(size_t n_, cudaStream_t s) : n(n_), stream(s) {
    if (n) check_cuda(cudaMallocAsync(reinterpret_cast<void**>(&ptr), n * sizeof(float), s), "tensor storage");
  }
  ~Storage() {
    if (ptr) cudaFreeAsync(ptr, stream);
  }
  Storage(const Storage&) = delete;
  Storage& operator=(const Storage&) = delete;
};
using Buf = std::shared_ptr<Storage>;

struct Node;
struct TensorImpl {
  uint64_t id = 0;
  std::vector<int64_t> shape;
  Buf data;
  bool requires_grad = false;  // a leaf whose gradient the caller wants
  std::shared_ptr<Node> node;  // the operation that made it, when it tracks gradients
  bool tracks() const { return requires_grad || node != nullptr; }
  long long numel() const {
    long long n = 1;
    for (int64_t d : shape) n *= d;
    return n;
  }
};
using T = std::shared_ptr<TensorImpl>;

// grad_of(i) gives parent i's gradient buffer (zero-filled on first use); the
// backward adds its contribution into it.
using GradOf = std::function<float*(size_t)>;
struct Node {
  std::vector<T> parents;
  std::function<void(const float* grad_out, const GradOf& grad_of)> backward;
};

struct Tape {
  int device = 0;
  int precision = MM_GPU_TF32;
  cudaStream_t stream = nullptr;
  uint64_t next_id = 1;
  std::unordered_map<uint64_t, T> handles;           // tensors the caller holds
  std::unordered_map<uint64_t, Buf> leaf_grads;      // after backward: gradients of requires_grad leaves
  std::map<std::tuple<int, int, float>, std::pair<Buf, Buf>> rope_cache;  // (head_dim, seq, theta)

  ~Tape() {
    handles.clear();
    leaf_grads.clear();
    rope_cache.clear();
    if (stream) {
      cudaStreamSynchronize(stream);
      cudaStreamDestroy(stream);
    }
  }

  Buf alloc(size_t n) { return std::make_shared<Storage>(n, stream); }
  Buf zeros(size_t n) {
    Buf b = alloc(n);
    if (n) check_cuda(cudaMemsetAsync(b->ptr, 0, n * sizeof(float), stream), "zero");
    return b;
  }
  Buf copy_of(const Buf& src) {
    Buf b = alloc(src->n);
    if (src->n) check_cuda(cudaMemcpyAsync(b->ptr, src->ptr, src->n * sizeof(float), cudaMemcpyDeviceToDevice, stream),
                           "copy");
    return b;
  }
  T make(std::vector<int64_t> shape, Buf data, std::vector<T> parents,
         std::function<void(const float*, const GradOf&)> backward) {
    auto t = std::make_shared<TensorImpl>();
    t->id = next_id++;
    t->shape = std::move(shape);
    t->data = std::move(data);
    bool any = false;
    for (const T& p : parents) any = any || p->tracks();
    if (any) {  // autograd.rs:27-41: a node only when some input tracks gradients
      t->node = std::make_shared<Node>();
      t->node->parents = std::move(parents);
      t->node->backward = std::move(backward);
    }
    handles[t->id] = t;
    return t;
  }
  T get(uint64_t h) const {
    auto it = handles.find(h);
    if (it == handles.end()) throw std::invalid_argument("tensor handle " + std::to_string(h) + " is not live");
    return it->second;
  }
  void gemm(int M, int N, int K, GemmOperand A, GemmOperand B, float* C, long long ldc, const float* R,
            long long ldr) {
    const int rc = precision == MM_GPU_TF32 ? gemm_tf32(M, N, K, A, B, C, ldc, R, ldr, device_context().d_err, stream)
                                            : gemm_3xtf32(M, N, K, A, B, C, ldc, R, ldr, device_context().d_err, stream);
    if (rc) throw std::runtime_error(std::string("matmul: ") + gemm_status_string(rc));
  }
  void add_into(float* dst, const float* src, long long n) { add(dst, src, dst, n, stream); }
  const std::pair<Buf, Buf>& rope_table(int hd, int seq, float theta) {
    auto key = std::make_tuple(hd, seq, theta);
    auto it = rope_cache.find(key);
    if (it != rope_cache.end()) return it->second;
    std::vector<float> c, s;
    ::mm::rope_tables(static_cast<uint64_t>(hd), static_cast<uint64_t>(seq), theta, c, s);
    Buf dc = alloc(c.size()), ds = alloc(s.size());
    check_cuda(cudaMemcpyAsync(dc->ptr, c.data(), c.size() * 4, cudaMemcpyHostToDevice, stream), "rope table");
    check_cuda(cudaMemcpyAsync(ds->ptr, s.data(), s.size() * 4, cudaMemcpyHostToDevice, stream), "rope table");
    check_cuda(cudaStreamSynchronize(stream), "rope table");  // the host vectors die here
    return rope_cache[key] = {dc, ds};
  }

  // Tensor::backward (autograd.rs:69-124) with device buffers.
  void backward(const T& root) {
    if (root->numel() != 1) throw std::invalid_argument("backward needs a single value");
    if (!root->tracks()) throw std::invalid_argument("backward called on a tensor that does not track gradients");
    std::vector<T> order;
    std::unordered_set<uint64_t> visited;
    std::vector<std::pair<T, bool>> stack{{root, false}};
    while (!stack.empty()) {
      auto [t, expanded] = stack.back();
      stack.pop_back();
      if (expanded) {
        order.push_back(t);
        continue;
      }
      if (!visited.insert(t->id).second) continue;
      stack.push_back({t, true});
      if (t->node)
        for (const T& p : t->node->parents)
          if (p->tracks() && !visited.count(p->id)) stack.push_back({p, false});
    }
    std::unordered_map<uint64_t, Buf> grads;
    Buf seed = alloc(1);
    fill_kernel<<<1, 32, 0, stream>>>(seed->ptr, 1.0f, 1);
    check_cuda(cudaGetLastError(), "seed");
    grads[root->id] = seed;
    for (auto it = order.rbegin(); it != order.rend(); ++it) {
      const T& t = *it;
      if (!t->node) continue;  // a leaf keeps its gradient
      auto g = grads.find(t->id);
      if (g == grads.end()) continue;  // nothing flowed into this node
      Buf grad_out = g->second;
      grads.erase(g);
      const Node& node = *t->node;
      GradOf grad_of = [&](size_t i) -> float* {
        const T& p = node.parents[i];
        if (!p->tracks()) return nullptr;
        Buf& b = grads[p->id];
        if (!b) b = zeros(static_cast<size_t>(p->numel()));
        return b->ptr;
      };
      node.backward(grad_out->ptr, grad_of);
    }
    for (auto& [id, b] : grads) leaf_grads[id] = b;  // what is left belongs to leaves
  }
};

std::mutex g_mu;
std::unordered_map<uint32_t, std::unique_ptr<Tape>> g_tapes;
uint32_t g_next_tape = 1;

Tape& tape_of(uint32_t h) {
  auto it = g_tapes.find(h);
  if (it == g_tapes.end()) throw std::invalid_argument("tape handle " + std::to_string(h) + " is not live");
  int dev = 0;
  check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  if (dev != it->second->device) throw std::invalid_argument("the tape belongs to another device");
  return *it->second;
}

struct ArgError : std::invalid_argument {
  int32_t code;
  ArgError(int32_t c, const std::string& m) : std::invalid_argument(m), code(c) {}
};

void require(bool ok, int32_t code, const std::string& msg) {
  if (!ok) throw ArgError(code, msg);
}

// Runs `body` under the tapes' lock; errors become status codes (or handle 0)
// with the message for mm_gpu_last_error.
template <class R, class F>
R guarded(R on_error, F&& body) {
  std::lock_guard<std::mutex> lock(g_mu);
  try {
    set_last_error("");
    return body();
  } catch (const ArgError& e) {
    set_last_error(e.what());
    return on_error == R(0) ? R(0) : static_cast<R>(e.code);
  } catch (const std::invalid_argument& e) {
    set_last_error(e.what());
    return on_error == R(0) ? R(0) : static_cast<R>(MM_GPU_ERR_ARGUMENT);
  } catch (const std::exception& e) {
    set_last_error(e.what());
    return on_error;
  }
}

bool multiple4(int64_t v) { return v % 4 == 0; }

}  // namespace
}  // namespace mm

using namespace mm;

extern "C" {

uint32_t mm_tape_create(int32_t precision) {
  return guarded<uint32_t>(0, [&]() -> uint32_t {
    require(precision == MM_GPU_TF32 || precision == MM_GPU_3XTF32, MM_GPU_ERR_ARGUMENT,
            "precision must be MM_GPU_TF32 or MM_GPU_3XTF32");
    auto t = std::make_unique<Tape>();
    check_cuda(cudaGetDevice(&t->device), "cudaGetDevice");
    t->precision = precision;
    check_cuda(cudaStreamCreateWithFlags(&t->stream, cudaStreamNonBlocking), "tape stream");
    const uint32_t h = g_next_tape++;
    g_tapes[h] = std::move(t);
    return h;
  });
}

int32_t mm_tape_destroy(uint32_t tape) {
  return guarded<int32_t>(MM_GPU_ERR_DEVICE, [&]() -> int32_t {
    tape_of(tape);
    g_tapes.erase(tape);
    return MM_GPU_OK;
  });
}

uint64_t mm_tensor_new(uint32_t tape, const int64_t* shape, int32_t rank, const float* host_values,
                       int32_t requires_grad) {
  return guarded<uint64_t>(0, [&]() -> uint64_t {
    Tape& tp = tape_of(tape);
    require(rank >= 1 && rank <= 4 && shape, MM_GPU_ERR_SHAPE, "tensor: rank 1 to 4 with its shape");
    std::vector<int64_t> sh(shape, shape + rank);
    long long n = 1;
    for (int64_t d : sh) {
      require(d > 0, MM_GPU_ERR_SHAPE, "tensor: dimensions must be positive");
      n *= d;
    }
    Buf b = host_values ? tp.alloc(static_cast<size_t>(n)) : tp.zeros(static_cast<size_t>(n));
    if (host_values) {
      check_cuda(cudaMemcpyAsync(b->ptr, host_values, n * sizeof(float), cudaMemcpyHostToDevice, tp.stream),
                 "tensor values");
      check_cuda(cudaStreamSynchronize(tp.stream), "tensor values");
    }
    T t = tp.make(sh, b, {}, nullptr);
    t->requires_grad = requires_grad != 0;
    return t->id;
  });
}

int32_t mm_tensor_shape(uint32_t tape, uint64_t tensor, int64_t* shape_out, int32_t* rank_out) {
  return guarded<int32_t>(MM_GPU_ERR_DEVICE, [&]() -> int32_t {
    T t = tape_of(tape).get(tensor);
    require(shape_out && rank_out, MM_GPU_ERR_ARGUMENT, "shape: null pointer");
    *rank_out = static_cast<int32_t>(t->shape.size());
    for (size_t i = 0; i < t->shape.size(); ++i) shape_out[i] = t->shape[i];
    return MM_GPU_OK;
  });
}

int32_t mm_tensor_read(uint32_t tape, uint64_t tensor, float* host_out, int64_t n) {
  return guarded<int32_t>(MM_GPU_ERR_DEVICE, [&]() -> int32_t {
    Tape& tp = tape_of(tape);
    T t = tp.get(tensor);
    require(host_out && n == t->numel(), MM_GPU_ERR_SHAPE, "read: the output must hold the tensor's values");
    check_cuda(cudaMemcpyAsync(host_out, t->data->ptr, n * sizeof(float), cudaMemcpyDeviceToHost, tp.stream), "read");
    check_cuda(cudaStreamSynchronize(tp.stream), "read");
    const int code = take_device_error(tp.stream);
    if (code) throw std::runtime_error(device_error_message(code));
    return MM_GPU_OK;
  });
}

int32_t mm_tensor_grad(uint32_t tape, uint64_t tensor, float* host_out, int64_t n) {
  return guarded<int32_t>(MM_GPU_ERR_DEVICE, [&]() -> int32_t {
    Tape& tp = tape_of(tape);
    T t = tp.get(tensor);
    require(host_out && n == t->numel(), MM_GPU_ERR_SHAPE, "grad: the output must hold the tensor's values");
    auto it = tp.leaf_grads.find(t->id);
    if (it == tp.leaf_grads.end()) {  // no gradient reached it: zeros (Grads::get gives None; here 0)
      std::memset(host_out, 0, n * sizeof(float));
      return MM_GPU_OK;
    }
    check_cuda(cudaMemcpyAsync(host_out, it->second->ptr, n * sizeof(float), cudaMemcpyDeviceToHost, tp.stream),
               "grad");
    check_cuda(cudaStreamSynchronize(tp.stream), "grad");
    return MM_GPU_OK;
  });
}

int32_t mm_tensor_free(uint32_t tape, uint64_t tensor) {
  return guarded<int32_t>(MM_GPU_ERR_DEVICE, [&]() -> int32_t {
    Tape& tp = tape_of(tape);
    tp.get(tensor);
    tp.handles.erase(tensor);
    tp.leaf_grads.erase(tensor);
    return MM_GPU_OK;
  });
}

int32_t mm_tape_backward(uint32_t tape, uint64_t loss) {
  return guarded<int32_t>(MM_GPU_ERR_DEVICE, [&]() -> int32_t {
    Tape& tp = tape_of(tape);
    tp.leaf_grads.clear();
    tp.backward(tp.get(loss));
    check_cuda(cudaStreamSynchronize(tp.stream), "backward");
    const int code = take_device_error(tp.stream);
    if (code) throw std::runtime_error(device_error_message(code));
    return MM_GPU_OK;
  });
}

// ---- operations

uint64_t mm_op_matmul(uint32_t tape, uint64_t a_h, uint64_t b_h, int32_t b_transposed) {
  return guarded<uint64_t>(0, [&]() -> uint64_t {
    Tape& tp = tape_of(tape);
    T a = tp.get(a_h), b = tp.get(b_h);
    require(a->shape.size() == 2 && b->shape.size() == 2, MM_GPU_ERR_SHAPE, "matmul: two 2-D tensors");
    const int64_t m = a->shape[0], k = a->shape[1];
    const int64_t n = b_transposed ? b->shape[0] : b->shape[1];
    require((b_transposed ? b->shape[1] : b->shape[0]) == k, MM_GPU_ERR_SHAPE, "matmul: inner dimensions differ");
    require(multiple4(k) && multiple4(n), MM_GPU_ERR_SHAPE, "matmul: inner and output widths must be multiples of 4");
    const bool bt = b_transposed != 0;
    Buf c = tp.alloc(static_cast<size_t>(m * n));
    // C = A B: A K-major (ld k); B(n, k) = B[k][n] (MN-major, ld n) or Bt[n][k] (K-major, ld k)
    tp.gemm(m, n, k, {a->data->ptr, k, false}, {b->data->ptr, bt ? k : n, !bt}, c->ptr, n, nullptr, 0);
    Tape* tpp = &tp;
    return tp.make({m, n}, c, {a, b}, [tpp, a, b, m, n, k, bt](const float* dc, const GradOf& grad_of) {
      // ops_matmul.rs:62-74: dA = dC B^T, dB = A^T dC (accumulated: R = the gradient so far)
      if (float* da = grad_of(0))
        tpp->gemm(m, k, n, {dc, n, false}, {b->data->ptr, bt ? k : n, bt}, da, k, da, k);
      if (float* db = grad_of(1)) {
        if (!bt)
          tpp->gemm(k, n, m, {a->data->ptr, k, true}, {dc, n, true}, db, n, db, n);
        else  // dBt = dC^T A  [n, k]
          tpp->gemm(n, k, m, {dc, n, true}, {a->data->ptr, k, true}, db, k, db, k);
      }
    })->id;
  });
}

uint64_t mm_op_add(uint32_t tape, uint64_t a_h, uint64_t b_h) {
  return guarded<uint64_t>(0, [&]() -> uint64_t {
    Tape& tp = tape_of(tape);
    T a = tp.get(a_h), b = tp.get(b_h);
    require(a->shape == b->shape, MM_GPU_ERR_SHAPE, "add: the shapes differ");
    const long long n = a->numel();
    Buf c = tp.alloc(static_cast<size_t>(n));
    add(a->data->ptr, b->data->ptr, c->ptr, n, tp.stream);
    Tape* tpp = &tp;
    return tp.make(a->shape, c, {a, b}, [tpp, n](const float* dc, const GradOf& grad_of) {
      for (size_t i = 0; i < 2; ++i)
        if (float* d = grad_of(i)) tpp->add_into(d, dc, n);
    })->id;
  });
}

uint64_t mm_op_mul(uint32_t tape, uint64_t a_h, uint64_t b_h) {
  return guarded<uint64_t>(0, [&]() -> uint64_t {
    Tape& tp = tape_of(tape);
    T a = tp.get(a_h), b = tp.get(b_h);
    require(a->shape == b->shape, MM_GPU_ERR_SHAPE, "mul: the shapes differ");
    const long long n = a->numel();
    Buf c = tp.alloc(static_cast<size_t>(n));
    mul_kernel<<<blocks_for(n), 256, 0, tp.stream>>>(a->data->ptr, b->data->ptr, c->ptr, n, 0);
    check_cuda(cudaGetLastError(), "mul");
    Tape* tpp = &tp;
    return tp.make(a->shape, c, {a, b}, [tpp, a, b, n](const float* dc, const GradOf& grad_of) {
      // ops_elementwise.rs:287: d a = g * b, d b = g * a
      if (float* da = grad_of(0)) mul_kernel<<<blocks_for(n), 256, 0, tpp->stream>>>(dc, b->data->ptr, da, n, 1);
      if (float* db = grad_of(1)) mul_kernel<<<blocks_for(n), 256, 0, tpp->stream>>>(dc, a->data->ptr, db, n, 1);
      check_cuda(cudaGetLastError(), "mul backward");
    })->id;
  });
}

uint64_t mm_op_embedding(uint32_t tape, uint64_t table_h, const int32_t* ids_host, int64_t rows) {
  return guarded<uint64_t>(0, [&]() -> uint64_t {
    Tape& tp = tape_of(tape);
    T table = tp.get(table_h);
    require(table->shape.size() == 2 && multiple4(table->shape[1]), MM_GPU_ERR_SHAPE,
            "embedding: a [vocab, dim] table with dim a multiple of 4");
    require(rows > 0 && ids_host, MM_GPU_ERR_ARGUMENT, "embedding: ids");
    const int vocab = static_cast<int>(table->shape[0]), dim = static_cast<int>(table->shape[1]);
    std::vector<int32_t> ids(ids_host, ids_host + rows);
    for (int64_t r = 0; r < rows; ++r)
      require(ids[r] >= 0 && ids[r] < vocab, MM_GPU_ERR_INDEX,
              "embedding: id " + std::to_string(ids[r]) + " is outside the table's " + std::to_string(vocab) + " rows");
    Buf d_ids = tp.alloc(static_cast<size_t>(rows));  // int32 ids, four bytes each like the floats
    check_cuda(cudaMemcpyAsync(d_ids->ptr, ids.data(), rows * 4, cudaMemcpyHostToDevice, tp.stream), "ids");
    Buf out = tp.alloc(static_cast<size_t>(rows) * dim);
    embedding_forward(reinterpret_cast<const int32_t*>(d_ids->ptr), static_cast<int>(rows), table->data->ptr, vocab,
                      dim, out->ptr, device_context().d_err, tp.stream);
    check_cuda(cudaStreamSynchronize(tp.stream), "ids");  // the host copy may go
    Tape* tpp = &tp;
    return tp.make({rows, dim}, out, {table}, [tpp, ids, vocab, dim](const float* dout, const GradOf& grad_of) {
      float* dt = grad_of(0);
      if (!dt) return;
      // ops_shape.rs:262-272: each table row adds its rows' gradients in row order
      std::vector<std::pair<int32_t, int32_t>> order(ids.size());
      for (size_t r = 0; r < ids.size(); ++r) order[r] = {ids[r], static_cast<int32_t>(r)};
      std::sort(order.begin(), order.end());
      std::vector<int32_t> uniq, offs, pos;
      for (size_t i = 0; i < order.size(); ++i) {
        if (i == 0 || order[i].first != order[i - 1].first) {
          uniq.push_back(order[i].first);
          offs.push_back(static_cast<int32_t>(i));
        }
        pos.push_back(order[i].second);
      }
      offs.push_back(static_cast<int32_t>(order.size()));
      std::vector<int32_t> csr(uniq);
      csr.insert(csr.end(), offs.begin(), offs.end());
      csr.insert(csr.end(), pos.begin(), pos.end());
      Buf d = tpp->alloc(csr.size());
      check_cuda(cudaMemcpyAsync(d->ptr, csr.data(), csr.size() * 4, cudaMemcpyHostToDevice, tpp->stream), "csr");
      const int32_t* di = reinterpret_cast<const int32_t*>(d->ptr);
      const int nu = static_cast<int>(uniq.size());
      embedding_backward(di, di + nu, di + 2 * nu + 1, nu, dout, dim, dt, tpp->stream);
      check_cuda(cudaStreamSynchronize(tpp->stream), "csr");  // the host index may go
      (void)vocab;
    })->id;
  });
}

uint64_t mm_op_rms_norm(uint32_t tape, uint64_t x_h, uint64_t w_h, float eps) {
  return guarded<uint64_t>(0, [&]() -> uint64_t {
    Tape& tp = tape_of(tape);
    T x = tp.get(x_h), w = tp.get(w_h);
    require(x->shape.size() == 2 && w->shape.size() == 1 && w->shape[0] == x->shape[1], MM_GPU_ERR_SHAPE,
            "rms_norm: x [rows, dim] and w [dim]");
    const int rows = static_cast<int>(x->shape[0]), dim = static_cast<int>(x->shape[1]);
    require(multiple4(dim) && dim <= 8192, MM_GPU_ERR_SHAPE, "rms_norm: dim a multiple of 4 up to 8192");
    Buf y = tp.alloc(static_cast<size_t>(rows) * dim), rstd = tp.alloc(rows);
    rmsnorm_forward(x->data->ptr, w->data->ptr, rows, dim, eps, y->ptr, rstd->ptr, tp.stream);
    Tape* tpp = &tp;
    return tp.make(x->shape, y, {x, w}, [tpp, x, w, rstd, rows, dim](const float* dy, const GradOf& grad_of) {
      float* dx = grad_of(0);
      float* dw = grad_of(1);
      Buf tmp_dx = dx ? Buf() : tpp->alloc(static_cast<size_t>(rows) * dim);
      Buf dw_part = tpp->alloc(dim);
      Buf ws = tpp->alloc(static_cast<size_t>(rmsnorm_ws_floats(rows, dim)));
      // dx (accumulated: dres = dx) and this use's dw, added into dw
      rmsnorm_backward(x->data->ptr, w->data->ptr, rstd->ptr, dy, rows, dim, dx ? dx : tmp_dx->ptr, dx, dw_part->ptr,
                       ws->ptr, tpp->stream);
      if (dw) tpp->add_into(dw, dw_part->ptr, dim);
    })->id;
  });
}

uint64_t mm_op_rope(uint32_t tape, uint64_t x_h, int32_t seq, int32_t heads, float theta) {
  return guarded<uint64_t>(0, [&]() -> uint64_t {
    Tape& tp = tape_of(tape);
    T x = tp.get(x_h);
    require(x->shape.size() == 2 && seq > 0 && heads > 0 && x->shape[0] % seq == 0 && x->shape[1] % heads == 0 &&
                (x->shape[1] / heads) % 2 == 0,
            MM_GPU_ERR_SHAPE, "rope: x [batch * seq, heads * head_dim] with an even head_dim");
    const int rows = static_cast<int>(x->shape[0]), hd = static_cast<int>(x->shape[1] / heads);
    const auto& tables = tp.rope_table(hd, seq, theta);
    Buf y = tp.copy_of(x->data);
    rope(y->ptr, rows, seq, heads, hd, x->shape[1], tables.first->ptr, tables.second->ptr, false, tp.stream);
    Tape* tpp = &tp;
    Buf c = tables.first, s = tables.second;
    const long long n = x->numel(), ld = x->shape[1];
    return tp.make(x->shape, y, {x}, [tpp, c, s, rows, seq, heads, hd, n, ld](const float* dy, const GradOf& grad_of) {
      float* dx = grad_of(0);
      if (!dx) return;
      Buf g = tpp->alloc(static_cast<size_t>(n));
      check_cuda(cudaMemcpyAsync(g->ptr, dy, n * 4, cudaMemcpyDeviceToDevice, tpp->stream), "rope backward");
      rope(g->ptr, rows, seq, heads, hd, ld, c->ptr, s->ptr, true, tpp->stream);  // rope.rs:114-132
      tpp->add_into(dx, g->ptr, n);
    })->id;
  });
}

uint64_t mm_op_causal_attention(uint32_t tape, uint64_t q_h, uint64_t k_h, uint64_t v_h, int32_t batch, int32_t seq,
                                int32_t n_heads, int32_t n_kv_heads) {
  return guarded<uint64_t>(0, [&]() -> uint64_t {
    Tape& tp = tape_of(tape);
    T q = tp.get(q_h), k = tp.get(k_h), v = tp.get(v_h);
    require(batch > 0 && seq > 0 && n_heads > 0 && n_kv_heads > 0 && n_heads % n_kv_heads == 0, MM_GPU_ERR_SHAPE,
            "attention: positive sizes, n_heads a multiple of n_kv_heads");
    require(q->shape.size() == 2 && q->shape[0] == static_cast<int64_t>(batch) * seq && q->shape[1] % n_heads == 0,
            MM_GPU_ERR_SHAPE, "attention: q [batch * seq, n_heads * head_dim]");
    const int hd = static_cast<int>(q->shape[1] / n_heads);
    require(k->shape == std::vector<int64_t>{q->shape[0], static_cast<int64_t>(n_kv_heads) * hd} && v->shape == k->shape,
            MM_GPU_ERR_SHAPE, "attention: k and v [batch * seq, n_kv_heads * head_dim]");
    require(hd <= 128 && hd % 2 == 0 && multiple4(q->shape[1]) && multiple4(k->shape[1]), MM_GPU_ERR_SHAPE,
            "attention: even head_dim up to 128, widths multiples of 4");
    const AttnShape s{batch, seq, n_heads, n_kv_heads, hd, q->shape[1], k->shape[1], k->shape[1], q->shape[1],
                      1.0f / std::sqrt(static_cast<float>(hd))};
    Buf o = tp.alloc(static_cast<size_t>(q->numel())), lse = tp.alloc(static_cast<size_t>(batch) * n_heads * seq);
    const bool flash = tp.precision == MM_GPU_TF32 && attention_flash_supported(s);
    const bool tc3 = tp.precision == MM_GPU_3XTF32 && attention_tc_supported(s);  // 3xTF32 on the tensor cores
    if (flash) {
      attention_forward_flash(s, q->data->ptr, k->data->ptr, v->data->ptr, o->ptr, lse->ptr, device_context().d_err,
                              tp.stream);
    } else if (tc3) {
      Buf ws = tp.alloc(static_cast<size_t>(attention_3x_ws_floats(s, s.ldo)));  // freed in stream order
      attention_forward_3x(s, q->data->ptr, k->data->ptr, v->data->ptr, o->ptr, lse->ptr, ws->ptr,
                           device_context().d_err, tp.stream);
    } else {
      attention_forward(s, q->data->ptr, k->data->ptr, v->data->ptr, o->ptr, lse->ptr, tp.stream);
    }
    Tape* tpp = &tp;
    return tp.make(q->shape, o, {q, k, v}, [tpp, q, k, v, o, lse, s, flash, tc3](const float* dout,
                                                                               const GradOf& grad_of) {
      Buf dq = tpp->alloc(static_cast<size_t>(q->numel())), dk = tpp->alloc(static_cast<size_t>(k->numel())),
          dv = tpp->alloc(static_cast<size_t>(v->numel()));
      Buf delta = tpp->alloc(static_cast<size_t>(s.B) * s.H * s.T);
      if (flash) {
        attention_backward_flash(s, q->data->ptr, k->data->ptr, v->data->ptr, o->ptr, lse->ptr, dout, s.ldo, dq->ptr,
                                 dk->ptr, dv->ptr, delta->ptr, device_context().d_err, tpp->stream);
      } else if (tc3) {
        Buf ws = tpp->alloc(static_cast<size_t>(attention_3x_ws_floats(s, s.ldo)));
        attention_backward_3x(s, q->data->ptr, k->data->ptr, v->data->ptr, o->ptr, lse->ptr, dout, s.ldo, dq->ptr, dk->ptr,
                              dv->ptr, ws->ptr, device_context().d_err, tpp->stream);
      } else {
        attention_backward(s, q->data->ptr, k->data->ptr, v->data->ptr, o->ptr, lse->ptr, dout, s.ldo, dq->ptr,
                           dk->ptr, dv->ptr, delta->ptr, tpp->stream);
      }
      const Buf parts[3] = {dq, dk, dv};
      for (size_t i = 0; i < 3; ++i)
        if (float* d = grad_of(i)) tpp->add_into(d, parts[i]->ptr, static_cast<long long>(parts[i]->n));
    })->id;
  });
}

uint64_t mm_op_swiglu(uint32_t tape, uint64_t gate_h, uint64_t up_h) {
  return guarded<uint64_t>(0, [&]() -> uint64_t {
    Tape& tp = tape_of(tape);
    T g = tp.get(gate_h), u = tp.get(up_h);
    require(g->shape == u->shape, MM_GPU_ERR_SHAPE, "swiglu: gate and up differ in shape");
    const long long n = g->numel();
    Buf act = tp.alloc(static_cast<size_t>(n));
    swiglu_forward(g->data->ptr, u->data->ptr, act->ptr, n, tp.stream);
    Tape* tpp = &tp;
    return tp.make(g->shape, act, {g, u}, [tpp, g, u, n](const float* dact, const GradOf& grad_of) {
      Buf dg = tpp->copy_of(g->data), du = tpp->copy_of(u->data);
      swiglu_backward(dg->ptr, du->ptr, dact, n, tpp->stream);  // in place: dgate, dup
      if (float* d = grad_of(0)) tpp->add_into(d, dg->ptr, n);
      if (float* d = grad_of(1)) tpp->add_into(d, du->ptr, n);
    })->id;
  });
}

uint64_t mm_op_cross_entropy(uint32_t tape, uint64_t logits_h, const int32_t* targets_host, int64_t rows) {
  return guarded<uint64_t>(0, [&]() -> uint64_t {
    Tape& tp = tape_of(tape);
    T z = tp.get(logits_h);
    require(z->shape.size() == 2 && z->shape[0] == rows && targets_host, MM_GPU_ERR_SHAPE,
            "cross_entropy: logits [rows, classes] and one target per row");
    const int vocab = static_cast<int>(z->shape[1]);
    for (int64_t r = 0; r < rows; ++r)
      require(targets_host[r] >= 0 && targets_host[r] < vocab, MM_GPU_ERR_INDEX,
              "cross_entropy: target " + std::to_string(targets_host[r]) + " is outside the " + std::to_string(vocab) +
                  " classes");
    // the kernel turns its logits into d(mean loss)/d logits: it works on a copy
    Buf grad = tp.copy_of(z->data);
    Buf tgt = tp.alloc(static_cast<size_t>(rows)), row_loss = tp.alloc(static_cast<size_t>(rows));
    Buf mean = tp.alloc(2), loss = tp.alloc(1);  // one double
    check_cuda(cudaMemcpyAsync(tgt->ptr, targets_host, rows * 4, cudaMemcpyHostToDevice, tp.stream), "targets");
    cross_entropy(grad->ptr, vocab, reinterpret_cast<const int32_t*>(tgt->ptr), static_cast<int>(rows), vocab,
                  1.0f / static_cast<float>(rows), row_loss->ptr, device_context().d_err, tp.stream);
    mean_loss(row_loss->ptr, static_cast<int>(rows), reinterpret_cast<double*>(mean->ptr), tp.stream);
    double_to_float_kernel<<<1, 1, 0, tp.stream>>>(reinterpret_cast<const double*>(mean->ptr), loss->ptr);
    check_cuda(cudaGetLastError(), "loss");
    check_cuda(cudaStreamSynchronize(tp.stream), "targets");  // the caller's targets may go
    Tape* tpp = &tp;
    const long long n = z->numel();
    return tp.make({1}, loss, {z}, [tpp, grad, n](const float* dl, const GradOf& grad_of) {
      // ops_reduce.rs:262-272: softmax - onehot, scaled by the upstream gradient / rows
      if (float* dz = grad_of(0)) {
        axpy_dev_kernel<<<blocks_for(n), 256, 0, tpp->stream>>>(dl, grad->ptr, dz, n);
        check_cuda(cudaGetLastError(), "cross_entropy backward");
      }
    })->id;
  });
}

}  // extern "C"
