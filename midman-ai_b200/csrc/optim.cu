// Global-norm clipping and AdamW over the flat parameter vector
// (crates/midman-optim/src/clip.rs:29-59, adamw.rs:141-217).
//
// The norm is a sum of squares in f64 (clip.rs:30): a fixed grid of blocks each
// reduces a fixed contiguous range, then one block adds the partials in order,
// so the norm is the same on every run and on every data-parallel rank. The
// update kernel reads the norm and the loss on the device and does nothing when
// either is not finite, which is the reference's validate-then-mutate rule
// (trainer.rs:194-199, clip.rs:49-51, adamw.rs:176-181) without a host round trip.
#include <cuda_runtime.h>

#include <cmath>
#include <stdexcept>
#include <string>

#include "kernels.h"

namespace mm {

namespace {

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ double block_sum_d(double v, double* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum_d(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  const int nw = (blockDim.x + 31) >> 5;
  double t = lane < nw ? red[lane] : 0.0;
  return warp_sum_d(t);
}

__global__ void sumsq_kernel(const float* __restrict__ g, long long n, double* __restrict__ partials, long long lo,
                             long long hi) {
  __shared__ double red[32];
  // Each block reduces one contiguous range; ranges start on 4-element boundaries.
  // A block whose range is not inside [lo, hi) writes 0 (another rank's share).
  const long long per = norm_block_elems(n);
  const long long beg = per * blockIdx.x;
  const long long end = beg + per < n ? beg + per : n;
  double s = 0.0;
  if (beg < end && beg >= lo && end <= hi) {
    const long long nvec = (end - beg) / 4;
    const float4* g4 = reinterpret_cast<const float4*>(g + beg);
    for (long long j = threadIdx.x; j < nvec; j += blockDim.x) {
      const float4 v = g4[j];
      s += static_cast<double>(v.x) * v.x + static_cast<double>(v.y) * v.y + static_cast<double>(v.z) * v.z +
           static_cast<double>(v.w) * v.w;
    }
    for (long long j = beg + nvec * 4 + threadIdx.x; j < end; j += blockDim.x) s += static_cast<double>(g[j]) * g[j];
  }
  s = block_sum_d(s, red);
  if (threadIdx.x == 0) partials[blockIdx.x] = s;
}

__global__ void finish_norm_kernel(const double* __restrict__ partials, int n, const double* __restrict__ loss,
                                   float max_norm, float* __restrict__ out) {
  __shared__ double red[32];
  double s = 0.0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) s += partials[i];
  s = block_sum_d(s, red);
  if (threadIdx.x == 0) {
    const float norm = static_cast<float>(sqrt(s));
    const bool ok = isfinite(norm) && (loss == nullptr || isfinite(static_cast<float>(*loss)));
    out[0] = norm;
    out[1] = (ok && norm > max_norm) ? max_norm / (norm + 1e-6f) : 1.0f;  // clip.rs:52-57
    out[2] = ok ? 1.0f : 0.0f;
  }
}

// One block per chunk (a chunk never spans two parameters).
// m and v hold the moments of elements [mv_base, ...) of the flat vector (the whole
// vector, or one rank's share of it under optimizer-state sharding).
__global__ void adamw_kernel(const AdamChunk* __restrict__ chunks, float* __restrict__ p, const float* __restrict__ g,
                             float* __restrict__ m, float* __restrict__ v, long long mv_base,
                             const float* __restrict__ norm_out, float lr, float beta1, float beta2, float eps,
                             float wd, float step_size, float bias2_sqrt) {
  if (norm_out[2] == 0.0f) return;  // a rejected step changes nothing
  const float factor = norm_out[1];
  const AdamChunk c = chunks[blockIdx.x];
  const float decay = c.decay ? 1.0f - lr * wd : 1.0f;
  const float omb1 = 1.0f - beta1, omb2 = 1.0f - beta2;
  const long long base = c.offset;
  m += base - mv_base;
  v += base - mv_base;
  for (int i = threadIdx.x * 4; i < c.length; i += blockDim.x * 4) {
    const long long k = base + i;
    const long long km = i;  // index into m and v
    if (i + 3 < c.length) {
      float4 x = *reinterpret_cast<float4*>(p + k);
      float4 gg = *reinterpret_cast<const float4*>(g + k);
      float4 mm_ = *reinterpret_cast<float4*>(m + km);
      float4 vv = *reinterpret_cast<float4*>(v + km);
      float* xs = &x.x;
      float* gs = &gg.x;
      float* ms = &mm_.x;
      float* vs = &vv.x;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float gr = gs[e] * factor;
        xs[e] *= decay;
        ms[e] = beta1 * ms[e] + omb1 * gr;
        vs[e] = beta2 * vs[e] + omb2 * gr * gr;
        xs[e] -= step_size * ms[e] / (sqrtf(vs[e]) / bias2_sqrt + eps);
      }
      *reinterpret_cast<float4*>(p + k) = x;
      *reinterpret_cast<float4*>(m + km) = mm_;
      *reinterpret_cast<float4*>(v + km) = vv;
    } else {
      for (int e = 0; e < 4 && i + e < c.length; ++e) {
        const float gr = g[k + e] * factor;
        float x = p[k + e] * decay;
        const float mn = beta1 * m[km + e] + omb1 * gr;
        const float vn = beta2 * v[km + e] + omb2 * gr * gr;
        x -= step_size * mn / (sqrtf(vn) / bias2_sqrt + eps);
        p[k + e] = x;
        m[km + e] = mn;
        v[km + e] = vn;
      }
    }
  }
}

__global__ void tensor_sumsq_kernel(const float* __restrict__ x, long long n, double* out) {
  __shared__ double red[32];
  double s = 0.0;
  for (long long i = threadIdx.x; i < n; i += blockDim.x) s += static_cast<double>(x[i]) * x[i];
  s = block_sum_d(s, red);
  if (threadIdx.x == 0) out[0] = s;
}

void check(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

}  // namespace

void sumsq_partials(const float* g, long long n, double* partials, cudaStream_t s, long long lo, long long hi) {
  sumsq_kernel<<<kNormBlocks, 256, 0, s>>>(g, n, partials, lo, hi < 0 ? n : hi);
  check("sumsq_partials");
}

void finish_norm(const double* partials, const double* loss, float max_norm, float* norm_out, cudaStream_t s) {
  finish_norm_kernel<<<1, 1024, 0, s>>>(partials, kNormBlocks, loss, max_norm, norm_out);
  check("finish_norm");
}

void adamw_step(const AdamChunk* chunks, int n_chunks, float* p, const float* g, float* m, float* v,
                long long mv_base, const float* norm_out, float lr, float beta1, float beta2, float eps,
                float weight_decay, float step_size, float bias2_sqrt, cudaStream_t s) {
  if (n_chunks <= 0) return;
  adamw_kernel<<<n_chunks, 256, 0, s>>>(chunks, p, g, m, v, mv_base, norm_out, lr, beta1, beta2, eps, weight_decay,
                                        step_size, bias2_sqrt);
  check("adamw_step");
}

void tensor_sumsq(const float* x, long long n, double* out, cudaStream_t s) {
  tensor_sumsq_kernel<<<1, 1024, 0, s>>>(x, n, out);
  check("tensor_sumsq");
}

}  // namespace mm
