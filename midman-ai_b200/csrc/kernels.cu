// Bandwidth-bound kernels of the training step: embedding, RMSNorm, RoPE,
// SwiGLU, softmax cross-entropy and the elementwise helpers. Each cites the
// reference function whose arithmetic it follows. Rows are processed by whole
// blocks with 128-bit accesses where the widths allow; reductions are tree
// reductions in a fixed order, so results are identical from run to run.
#include <cuda_runtime.h>

#include <cfloat>
#include <cmath>
#include <cstdint>
#include <stdexcept>

#include "kernels.h"

namespace mm {

namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Sum over the block; every thread gets the result. `red` holds 32 floats.
__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  const int nw = (blockDim.x + 31) >> 5;
  float t = lane < nw ? red[lane] : 0.0f;
  return warp_sum(t);
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

int grid_for(long long n, int per_thread = 4) {
  long long b = (n + static_cast<long long>(kThreads) * per_thread - 1) / (static_cast<long long>(kThreads) * per_thread);
  if (b < 1) b = 1;
  if (b > 148 * 64) b = 148 * 64;
  return static_cast<int>(b);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

void check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

// ---------------------------------------------------------------- embedding
// An id outside [0, vocab) reads nothing: its row is zero and the error flag
// gets kErrIndex (the reference refuses such ids, ops_shape.rs:238-244).
__global__ void embedding_fwd_kernel(const int32_t* __restrict__ ids, const float* __restrict__ table, int vocab,
                                     int dim, float* __restrict__ out, int* err) {
  const int r = blockIdx.x;
  const int id = ids[r];
  float4* dst = reinterpret_cast<float4*>(out + static_cast<long long>(r) * dim);
  if (id < 0 || id >= vocab) {
    for (int j = threadIdx.x; j < dim / 4; j += blockDim.x) dst[j] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (threadIdx.x == 0 && err) atomicCAS(err, 0, 7 /* kErrIndex */);
    return;
  }
  const float4* src = reinterpret_cast<const float4*>(table + static_cast<long long>(id) * dim);
  for (int j = threadIdx.x; j < dim / 4; j += blockDim.x) dst[j] = src[j];
}

// One block per distinct id: the existing row plus the positions' rows in
// ascending position order (ops_shape.rs:262-272 adds them in that order).
__global__ void embedding_bwd_kernel(const int32_t* __restrict__ uniq, const int32_t* __restrict__ offsets,
                                     const int32_t* __restrict__ positions, const float* __restrict__ dx, int dim,
                                     float* __restrict__ dtable) {
  const int u = blockIdx.x;
  const int beg = offsets[u], end = offsets[u + 1];
  float* row = dtable + static_cast<long long>(uniq[u]) * dim;
  for (int j = threadIdx.x; j < dim; j += blockDim.x) {
    float acc = row[j];
    for (int p = beg; p < end; ++p) acc += dx[static_cast<long long>(positions[p]) * dim + j];
    row[j] = acc;
  }
}

// ---------------------------------------------------------------- RMSNorm
// One block per row; the row stays in registers (G float4 per thread) between
// the sum of squares and the scaled write.
template <int G>
__global__ void rmsnorm_fwd_kernel(const float* __restrict__ x, const float* __restrict__ w, int dim, float eps,
                                   float* __restrict__ y, float* __restrict__ rstd) {
  __shared__ float red[32];
  const long long r = blockIdx.x;
  const int nv = dim / 4;
  const float4* xr = reinterpret_cast<const float4*>(x + r * dim);
  const float4* w4 = reinterpret_cast<const float4*>(w);
  float4* yr = reinterpret_cast<float4*>(y + r * dim);
  float4 v[G];
  float ss = 0.0f;
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const int j = threadIdx.x + g * blockDim.x;
    v[g] = j < nv ? xr[j] : make_float4(0.f, 0.f, 0.f, 0.f);
    ss += v[g].x * v[g].x + v[g].y * v[g].y + v[g].z * v[g].z + v[g].w * v[g].w;
  }
  ss = block_sum(ss, red);
  // mean_axis = sum * (1/len) (ops_reduce.rs:87-90), + eps, ^(-1/2)
  const float t = ss * (1.0f / static_cast<float>(dim)) + eps;
  const float inv = 1.0f / sqrtf(t);
  if (threadIdx.x == 0) rstd[r] = inv;
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const int j = threadIdx.x + g * blockDim.x;
    if (j < nv) {
      const float4 gw = w4[j];
      yr[j] = make_float4((v[g].x * inv) * gw.x, (v[g].y * inv) * gw.y, (v[g].z * inv) * gw.z,
                          (v[g].w * inv) * gw.w);
    }
  }
}

// Each block owns a contiguous range of rows; per row it writes dx and keeps the
// row's contribution to dw in registers (G float4 column groups per thread).
template <int G>
__global__ void __launch_bounds__(kThreads, G <= 2 ? 4 : 1)
    rmsnorm_bwd_kernel(const float* __restrict__ x, const float* __restrict__ w, const float* __restrict__ rstd,
                       const float* __restrict__ dy, int rows, int dim, int rows_per_block, float* dx,
                       const float* dres, float* __restrict__ ws) {
  __shared__ float red[32];
  const int r0 = blockIdx.x * rows_per_block;
  const int r1 = min(rows, r0 + rows_per_block);
  const int nv = dim / 4;
  const float4* w4 = reinterpret_cast<const float4*>(w);
  float4 acc[G];
#pragma unroll
  for (int g = 0; g < G; ++g) acc[g] = make_float4(0.f, 0.f, 0.f, 0.f);
  // the weights are read per row from L1 (registers go to the prefetched rows)
  auto wv = [&](int g) {
    const int j = threadIdx.x + g * blockDim.x;
    return j < nv ? __ldg(w4 + j) : make_float4(0.f, 0.f, 0.f, 0.f);
  };
  const float inv_dim = 1.0f / static_cast<float>(dim);
  // x, dy, the residual gradient and 1/rms of row r + 1 are loaded while row r
  // is reduced and written (rows differ, so dx may alias dy or dres)
  float4 xv[G], gv[G], dv[G], xn[G], gn[G], dn[G];
  float iv = 0.0f, in_ = 0.0f;
  auto load_row = [&](int r, float4 (&xa)[G], float4 (&ga)[G], float4 (&da)[G], float& ia) {
    const float4* xr = reinterpret_cast<const float4*>(x + static_cast<long long>(r) * dim);
    const float4* gr = reinterpret_cast<const float4*>(dy + static_cast<long long>(r) * dim);
    const float4* dr = dres ? reinterpret_cast<const float4*>(dres + static_cast<long long>(r) * dim) : nullptr;
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const int j = threadIdx.x + g * blockDim.x;
      xa[g] = j < nv ? xr[j] : make_float4(0.f, 0.f, 0.f, 0.f);
      ga[g] = j < nv ? gr[j] : make_float4(0.f, 0.f, 0.f, 0.f);
      da[g] = (dr && j < nv) ? dr[j] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    ia = rstd[r];
  };
  if (r0 < r1) load_row(r0, xv, gv, dv, iv);
  for (int r = r0; r < r1; ++r) {
    if (r + 1 < r1) load_row(r + 1, xn, gn, dn, in_);
    float dot = 0.0f;
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const int j = threadIdx.x + g * blockDim.x;
      if (j < nv) {
        const float4 wg = wv(g);
        dot += (gv[g].x * wg.x) * xv[g].x + (gv[g].y * wg.y) * xv[g].y + (gv[g].z * wg.z) * xv[g].z +
               (gv[g].w * wg.w) * xv[g].w;
      }
    }
    dot = block_sum(dot, red);
    const float inv = iv;
    // d/dx of x*inv*w through inv = (mean(x^2)+eps)^-1/2: the powf closure gives
    // -0.5*t^-1.5 = -0.5*inv^3, the mean's 1/len, and x*x contributes twice.
    const float dsum = (dot * (-0.5f * inv * inv * inv)) * inv_dim;
    float4* dxr = reinterpret_cast<float4*>(dx + static_cast<long long>(r) * dim);
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const int j = threadIdx.x + g * blockDim.x;
      if (j < nv) {
        const float4 b = make_float4(dsum * xv[g].x, dsum * xv[g].y, dsum * xv[g].z, dsum * xv[g].w);
        const float4 wg = wv(g);
        float4 o = make_float4(((gv[g].x * wg.x) * inv + b.x) + b.x, ((gv[g].y * wg.y) * inv + b.y) + b.y,
                               ((gv[g].z * wg.z) * inv + b.z) + b.z, ((gv[g].w * wg.w) * inv + b.w) + b.w);
        if (dres) {
          o.x += dv[g].x; o.y += dv[g].y; o.z += dv[g].z; o.w += dv[g].w;
        }
        dxr[j] = o;
        acc[g].x += gv[g].x * (xv[g].x * inv);
        acc[g].y += gv[g].y * (xv[g].y * inv);
        acc[g].z += gv[g].z * (xv[g].z * inv);
        acc[g].w += gv[g].w * (xv[g].w * inv);
      }
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
      xv[g] = xn[g];
      gv[g] = gn[g];
      dv[g] = dn[g];
    }
    iv = in_;
  }
  float4* out = reinterpret_cast<float4*>(ws + static_cast<long long>(blockIdx.x) * dim);
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const int j = threadIdx.x + g * blockDim.x;
    if (j < nv) out[j] = acc[g];
  }
}

// dw[j] = sum over the blocks' partial rows. A block owns 32 columns; each of
// its 32 warps sums rows w, w + 32, ... (coalesced 128-byte row segments) with
// four interleaved accumulators and eight loads in flight, and the warp sums
// are added in warp order, so the result does not depend on timing.
__global__ void __launch_bounds__(1024) column_sum_kernel(const float* __restrict__ ws, int nblk, int dim,
                                                          float* __restrict__ dw) {
  __shared__ float part[32][33];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int j = blockIdx.x * 32 + lane;
  float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
  if (j < dim) {
    const float* col = ws + j;
    const long long st = static_cast<long long>(dim);
    int b = warp;
#pragma unroll 2
    for (; b + 96 < nblk; b += 128) {
      a0 += col[b * st];
      a1 += col[(b + 32) * st];
      a2 += col[(b + 64) * st];
      a3 += col[(b + 96) * st];
    }
    for (; b < nblk; b += 32) a0 += col[b * st];
  }
  part[warp][lane] = (a0 + a1) + (a2 + a3);
  __syncthreads();
  if (warp == 0 && j < dim) {
    float s = 0.0f;
#pragma unroll
    for (int w = 0; w < 32; ++w) s += part[w][lane];
    dw[j] = s;
  }
}

int rmsnorm_bwd_blocks(int rows) { return rows < 592 ? rows : 592; }

// ---------------------------------------------------------------- RoPE
__global__ void rope_kernel(float* x, int rows, int T, int heads, int half, long long ld,
                            const float* __restrict__ cos_t, const float* __restrict__ sin_t, float sign) {
  const long long total = static_cast<long long>(rows) * heads * half;
  for (long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int i = static_cast<int>(idx % half);
    const long long rh = idx / half;
    const int h = static_cast<int>(rh % heads);
    const long long r = rh / heads;
    const int t = static_cast<int>(r % T);
    float* v = x + r * ld + static_cast<long long>(h) * 2 * half;
    const float c = cos_t[t * half + i], s = sign * sin_t[t * half + i];
    const float x1 = v[i], x2 = v[i + half];
    // forward (rope.rs:30-31): (x1 c - x2 s, x2 c + x1 s); gradient: s -> -s
    v[i] = x1 * c - x2 * s;
    v[i + half] = x2 * c + x1 * s;
  }
}

// Four consecutive i per thread (half % 4 == 0, 16-byte aligned rows and tables).
// One block per row (token): thread j of the row's heads * half / 4 handles
// four pairs (x[i], x[i + half]) of one head; the row's position picks the table row.
__global__ void rope4_kernel(float* x, int T, int heads, int half, long long ld, const float* __restrict__ cos_t,
                             const float* __restrict__ sin_t, float sign) {
  const int q4 = half / 4;
  const long long r = blockIdx.x;
  const int t = static_cast<int>(r % T);
  const float* ct = cos_t + static_cast<long long>(t) * half;
  const float* st = sin_t + static_cast<long long>(t) * half;
  float* row = x + r * ld;
  for (int j = threadIdx.x; j < heads * q4; j += blockDim.x) {
    const int h = j / q4, i = (j - h * q4) * 4;
    float* v = row + static_cast<long long>(h) * 2 * half;
    const float4 c = *reinterpret_cast<const float4*>(ct + i);
    const float4 sn = *reinterpret_cast<const float4*>(st + i);
    const float4 a = *reinterpret_cast<const float4*>(v + i), b = *reinterpret_cast<const float4*>(v + i + half);
    const float s0 = sign * sn.x, s1 = sign * sn.y, s2 = sign * sn.z, s3 = sign * sn.w;
    *reinterpret_cast<float4*>(v + i) =
        make_float4(a.x * c.x - b.x * s0, a.y * c.y - b.y * s1, a.z * c.z - b.z * s2, a.w * c.w - b.w * s3);
    *reinterpret_cast<float4*>(v + i + half) =
        make_float4(b.x * c.x + a.x * s0, b.y * c.y + a.y * s1, b.z * c.z + a.z * s2, b.w * c.w + a.w * s3);
  }
}

// ---------------------------------------------------------------- SwiGLU
__device__ __forceinline__ float sigmoidf_ref(float x) { return 1.0f / (1.0f + expf(-x)); }

__global__ void swiglu_fwd_kernel(const float* __restrict__ g, const float* __restrict__ u, float* __restrict__ act,
                                  long long n) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const float x = g[i];
    act[i] = (x * sigmoidf_ref(x)) * u[i];  // silu (ops_elementwise.rs:355-364) then mul
  }
}

// The same arithmetic per element, four elements per thread with 128-bit accesses.
__device__ __forceinline__ float silu_mul(float x, float up) { return (x * sigmoidf_ref(x)) * up; }

__global__ void swiglu_fwd4_kernel(const float4* __restrict__ g, const float4* __restrict__ u,
                                   float4* __restrict__ act, long long n4) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const float4 x = g[i], up = u[i];
    act[i] = make_float4(silu_mul(x.x, up.x), silu_mul(x.y, up.y), silu_mul(x.z, up.z), silu_mul(x.w, up.w));
  }
}

__device__ __forceinline__ void swiglu_grad1(float x, float up, float d, float& dg, float& du) {
  const float s = sigmoidf_ref(x);
  const float silu = x * s;
  dg = (d * up) * (s * (1.0f + x * (1.0f - s)));
  du = d * silu;
}

__global__ void swiglu_bwd4_kernel(float4* g, float4* u, const float4* __restrict__ dact, long long n4) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const float4 x = g[i], up = u[i], d = dact[i];
    float4 dg, du;
    swiglu_grad1(x.x, up.x, d.x, dg.x, du.x);
    swiglu_grad1(x.y, up.y, d.y, dg.y, du.y);
    swiglu_grad1(x.z, up.z, d.z, dg.z, du.z);
    swiglu_grad1(x.w, up.w, d.w, dg.w, du.w);
    g[i] = dg;
    u[i] = du;
  }
}

__global__ void swiglu_bwd_kernel(float* g, float* u, const float* __restrict__ dact, long long n) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const float x = g[i], up = u[i], d = dact[i];
    const float s = sigmoidf_ref(x);
    const float silu = x * s;
    g[i] = (d * up) * (s * (1.0f + x * (1.0f - s)));
    u[i] = d * silu;
  }
}

// ---------------------------------------------------------------- cross-entropy
struct MaxSum {
  float m, s;
};

__device__ __forceinline__ MaxSum combine(MaxSum a, MaxSum b) {
  if (a.m == -INFINITY) return b;
  if (b.m == -INFINITY) return a;
  const float m = fmaxf(a.m, b.m);
  return {m, a.s * expf(a.m - m) + b.s * expf(b.m - m)};
}

// A target outside [0, vocab) reads no logit: the row's loss is NaN, its
// gradient row is the softmax alone, and the error flag gets kErrIndex.
__global__ void cross_entropy_kernel(float* logits, long long ld, const int32_t* __restrict__ targets, int vocab,
                                     float grad_scale, float* __restrict__ row_loss, int* err) {
  __shared__ float sm[32], ss[32];
  __shared__ float row_max, row_sum;
  const long long r = blockIdx.x;
  float* z = logits + r * ld;
  const int t_raw = targets[r];
  const bool t_ok = t_raw >= 0 && t_raw < vocab;
  if (!t_ok && threadIdx.x == 0 && err) atomicCAS(err, 0, 7 /* kErrIndex */);
  MaxSum acc{-INFINITY, 0.0f};
  const bool vec = (vocab & 3) == 0 && (ld & 3) == 0 && (reinterpret_cast<uintptr_t>(logits) & 15u) == 0;
  if (vec) {  // four logits per step: one max update, then four exponentials against it
    const float4* z4 = reinterpret_cast<const float4*>(z);
    for (int j = threadIdx.x; j < vocab / 4; j += blockDim.x) {
      const float4 v = z4[j];
      const float m4 = fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w));
      if (m4 > acc.m) {
        acc.s = acc.m == -INFINITY ? 0.0f : acc.s * expf(acc.m - m4);
        acc.m = m4;
      }
      acc.s += (expf(v.x - acc.m) + expf(v.y - acc.m)) + (expf(v.z - acc.m) + expf(v.w - acc.m));
    }
  } else {
    for (int j = threadIdx.x; j < vocab; j += blockDim.x) {
      const float v = z[j];
      if (v > acc.m) {
        acc.s = (acc.m == -INFINITY ? 0.0f : acc.s * expf(acc.m - v)) + 1.0f;
        acc.m = v;
      } else {
        acc.s += expf(v - acc.m);
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    MaxSum other{__shfl_xor_sync(0xffffffffu, acc.m, o), __shfl_xor_sync(0xffffffffu, acc.s, o)};
    acc = combine(acc, other);
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) {
    sm[warp] = acc.m;
    ss[warp] = acc.s;
  }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    MaxSum a = lane < nw ? MaxSum{sm[lane], ss[lane]} : MaxSum{-INFINITY, 0.0f};
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      MaxSum other{__shfl_xor_sync(0xffffffffu, a.m, o), __shfl_xor_sync(0xffffffffu, a.s, o)};
      a = combine(a, other);
    }
    if (lane == 0) {
      row_max = a.m;
      row_sum = a.s;
      row_loss[r] = t_ok ? a.m + logf(a.s) - z[t_raw] : NAN;  // ops_reduce.rs:256-258
    }
  }
  __syncthreads();
  const float mx = row_max, sum = row_sum;
  const int t = t_ok ? t_raw : -1;
  // softmax * grad_scale as one multiply per logit: exp(v - max) * (grad_scale / sum).
  // The reference divides each exponential by the sum and then scales
  // (ops_reduce.rs:266-270); the product differs from that by at most an ulp or
  // two, and a division per logit made this pass instruction-bound.
  const float coef = grad_scale / sum;
  if (vec) {
    float4* z4 = reinterpret_cast<float4*>(z);
    for (int j = threadIdx.x; j < vocab / 4; j += blockDim.x) {
      const float4 v = z4[j];
      float4 d = make_float4(expf(v.x - mx) * coef, expf(v.y - mx) * coef, expf(v.z - mx) * coef,
                             expf(v.w - mx) * coef);
      if ((t >> 2) == j) {
        if ((t & 3) == 0) d.x -= grad_scale;
        if ((t & 3) == 1) d.y -= grad_scale;
        if ((t & 3) == 2) d.z -= grad_scale;
        if ((t & 3) == 3) d.w -= grad_scale;
      }
      z4[j] = d;
    }
  } else {
    for (int j = threadIdx.x; j < vocab; j += blockDim.x) {
      float d = expf(z[j] - mx) * coef;
      if (j == t) d -= grad_scale;
      z[j] = d;
    }
  }
}

__global__ void mean_loss_kernel(const float* __restrict__ row_loss, int rows, double* out) {
  __shared__ double red[32];
  double s = 0.0;
  for (int i = threadIdx.x; i < rows; i += blockDim.x) s += static_cast<double>(row_loss[i]);
  s = block_sum_d(s, red);
  if (threadIdx.x == 0) out[0] = s / static_cast<double>(rows);
}

__global__ void argmax_kernel(const float* __restrict__ logits, long long ld, int vocab, int32_t* out) {
  __shared__ float bv[32];
  __shared__ int bi[32];
  const float* z = logits + blockIdx.x * ld;
  float best = -INFINITY;
  int idx = 0x7fffffff;
  for (int j = threadIdx.x; j < vocab; j += blockDim.x) {
    const float v = z[j];
    if (v > best || (v == best && j < idx)) {
      best = v;
      idx = j;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (ov > best || (ov == best && oi < idx)) {
      best = ov;
      idx = oi;
    }
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) {
    bv[warp] = best;
    bi[warp] = idx;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float b = bv[0];
    int i = bi[0];
    for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w)
      if (bv[w] > b || (bv[w] == b && bi[w] < i)) {
        b = bv[w];
        i = bi[w];
      }
    out[blockIdx.x] = i == 0x7fffffff ? 0 : i;
  }
}

// ---------------------------------------------------------------- misc
__global__ void add_kernel(const float* a, const float* b, float* out, long long n) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x)
    out[i] = a[i] + b[i];
}

__global__ void scale_kernel(float* x, float f, long long n) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x)
    x[i] *= f;
}

}  // namespace

void embedding_forward(const int32_t* ids, int rows, const float* table, int vocab, int dim, float* out, int* err,
                       cudaStream_t s) {
  if (rows <= 0) return;
  embedding_fwd_kernel<<<rows, 128, 0, s>>>(ids, table, vocab, dim, out, err);
  check_launch("embedding_forward");
}

void embedding_backward(const int32_t* uniq, const int32_t* offsets, const int32_t* positions, int n_uniq,
                        const float* dx, int dim, float* dtable, cudaStream_t s) {
  if (n_uniq <= 0) return;
  embedding_bwd_kernel<<<n_uniq, 256, 0, s>>>(uniq, offsets, positions, dx, dim, dtable);
  check_launch("embedding_backward");
}

void rmsnorm_forward(const float* x, const float* w, int rows, int dim, float eps, float* y, float* rstd,
                     cudaStream_t s) {
  if (rows <= 0) return;
  const int groups = (dim / 4 + kThreads - 1) / kThreads;
  if (groups <= 1)
    rmsnorm_fwd_kernel<1><<<rows, kThreads, 0, s>>>(x, w, dim, eps, y, rstd);
  else if (groups <= 2)
    rmsnorm_fwd_kernel<2><<<rows, kThreads, 0, s>>>(x, w, dim, eps, y, rstd);
  else if (groups <= 4)
    rmsnorm_fwd_kernel<4><<<rows, kThreads, 0, s>>>(x, w, dim, eps, y, rstd);
  else if (groups <= 8)
    rmsnorm_fwd_kernel<8><<<rows, kThreads, 0, s>>>(x, w, dim, eps, y, rstd);
  else
    throw std::runtime_error("rmsnorm_forward: d_model above 8192 is not supported");
  check_launch("rmsnorm_forward");
}

long long rmsnorm_ws_floats(int rows, int dim) { return static_cast<long long>(rmsnorm_bwd_blocks(rows)) * dim; }

void rmsnorm_backward(const float* x, const float* w, const float* rstd, const float* dy, int rows, int dim,
                      float* dx, const float* dres, float* dw, float* ws, cudaStream_t s) {
  if (rows <= 0) return;
  const int nblk = rmsnorm_bwd_blocks(rows);
  const int rpb = (rows + nblk - 1) / nblk;
  const int groups = (dim / 4 + kThreads - 1) / kThreads;
  if (groups <= 1)
    rmsnorm_bwd_kernel<1><<<nblk, kThreads, 0, s>>>(x, w, rstd, dy, rows, dim, rpb, dx, dres, ws);
  else if (groups <= 2)
    rmsnorm_bwd_kernel<2><<<nblk, kThreads, 0, s>>>(x, w, rstd, dy, rows, dim, rpb, dx, dres, ws);
  else if (groups <= 4)
    rmsnorm_bwd_kernel<4><<<nblk, kThreads, 0, s>>>(x, w, rstd, dy, rows, dim, rpb, dx, dres, ws);
  else if (groups <= 8)
    rmsnorm_bwd_kernel<8><<<nblk, kThreads, 0, s>>>(x, w, rstd, dy, rows, dim, rpb, dx, dres, ws);
  else
    throw std::runtime_error("rmsnorm_backward: d_model above 8192 is not supported");
  check_launch("rmsnorm_backward");
  column_sum_kernel<<<(dim + 31) / 32, 1024, 0, s>>>(ws, nblk, dim, dw);
  check_launch("rmsnorm_backward(column sum)");
}

void rope(float* x, int rows, int T, int heads, int hd, long long ld, const float* cos_t, const float* sin_t,
          bool backward, cudaStream_t s) {
  const long long total = static_cast<long long>(rows) * heads * (hd / 2);
  if (total <= 0) return;
  const bool vec = (hd / 2) % 4 == 0 && ld % 4 == 0 && aligned16(x) && aligned16(cos_t) && aligned16(sin_t);
  if (vec) {
    const int per_row = heads * (hd / 8);  // float4 pairs per row
    const int threads = per_row >= 1024 ? 1024 : (per_row + 31) / 32 * 32;
    rope4_kernel<<<rows, threads, 0, s>>>(x, T, heads, hd / 2, ld, cos_t, sin_t, backward ? -1.0f : 1.0f);
  } else {
    rope_kernel<<<grid_for(total, 1), kThreads, 0, s>>>(x, rows, T, heads, hd / 2, ld, cos_t, sin_t,
                                                         backward ? -1.0f : 1.0f);
  }
  check_launch("rope");
}

void swiglu_forward(const float* g, const float* u, float* act, long long n, cudaStream_t s) {
  if (n <= 0) return;
  if (n % 4 == 0 && aligned16(g) && aligned16(u) && aligned16(act))
    swiglu_fwd4_kernel<<<grid_for(n / 4, 2), kThreads, 0, s>>>(reinterpret_cast<const float4*>(g),
                                                               reinterpret_cast<const float4*>(u),
                                                               reinterpret_cast<float4*>(act), n / 4);
  else
    swiglu_fwd_kernel<<<grid_for(n, 4), kThreads, 0, s>>>(g, u, act, n);
  check_launch("swiglu_forward");
}

void swiglu_backward(float* g, float* u, const float* dact, long long n, cudaStream_t s) {
  if (n <= 0) return;
  if (n % 4 == 0 && aligned16(g) && aligned16(u) && aligned16(dact))
    swiglu_bwd4_kernel<<<grid_for(n / 4, 2), kThreads, 0, s>>>(reinterpret_cast<float4*>(g),
                                                               reinterpret_cast<float4*>(u),
                                                               reinterpret_cast<const float4*>(dact), n / 4);
  else
    swiglu_bwd_kernel<<<grid_for(n, 4), kThreads, 0, s>>>(g, u, dact, n);
  check_launch("swiglu_backward");
}

void cross_entropy(float* logits, long long ld, const int32_t* targets, int rows, int vocab, float grad_scale,
                   float* row_loss, int* err, cudaStream_t s) {
  if (rows <= 0) return;
  const int threads = vocab >= 8192 ? 1024 : 256;
  cross_entropy_kernel<<<rows, threads, 0, s>>>(logits, ld, targets, vocab, grad_scale, row_loss, err);
  check_launch("cross_entropy");
}

void mean_loss(const float* row_loss, int rows, double* loss_out, cudaStream_t s) {
  mean_loss_kernel<<<1, 1024, 0, s>>>(row_loss, rows, loss_out);
  check_launch("mean_loss");
}

void argmax_rows(const float* logits, long long ld, int rows, int vocab, int32_t* out, cudaStream_t s) {
  if (rows <= 0) return;
  argmax_kernel<<<rows, 256, 0, s>>>(logits, ld, vocab, out);
  check_launch("argmax_rows");
}

void add(const float* a, const float* b, float* out, long long n, cudaStream_t s) {
  if (n <= 0) return;
  add_kernel<<<grid_for(n, 4), kThreads, 0, s>>>(a, b, out, n);
  check_launch("add");
}

void scale(float* x, float factor, long long n, cudaStream_t s) {
  if (n <= 0) return;
  scale_kernel<<<grid_for(n, 4), kThreads, 0, s>>>(x, factor, n);
  check_launch("scale");
}

}  // namespace mm
