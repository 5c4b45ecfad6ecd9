// 3xTF32 ("exact") mode of the GEMM: each operand is split into two TF32
// numbers, x ~ hi + lo with hi = x rounded to TF32 (nearest) and lo = (x - hi)
// rounded to TF32 as well, and the product is formed as hi*hi + hi*lo + lo*hi
// on the TF32 tensor cores (lo*lo is below f32 resolution). This is the split
// of Ootomo & Yokota (2022); rounding both parts to nearest (rather than
// truncating hi and letting the tensor core truncate lo) leaves
// |x - hi - lo| <= 2^-22 |x|, close to f32's own 2^-24, at 3x the MMA work.
#include <cuda_runtime.h>

#include <cstdint>

#include "device.h"
#include "gemm.h"

namespace mm {

namespace {

// Round to the nearest TF32 value (ties away from zero); the result's low 13
// mantissa bits are zero, so the tensor core reads it unchanged.
__device__ __forceinline__ float to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

__global__ void split_tf32_kernel(const float* __restrict__ x, float* __restrict__ hi,
                                  float* __restrict__ lo, long long n) {
  long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (; i < n; i += stride) {
    const float v = x[i];
    const float h = to_tf32(v);
    hi[i] = h;
    lo[i] = to_tf32(v - h);  // v - h is exact in f32; its TF32 rounding drops < 2^-11 of it
  }
}

// The part of x below its TF32 value as the tensor core reads x (the 19 high
// bits, the low 13 mantissa bits ignored), rounded to TF32 (nearest): a
// kind::tf32 product of x itself and of this lo together see x to within
// 2^-11 |x - trunc(x)| <= 2^-21 |x|, with no hi copy.
__global__ void split_lo_kernel(const float* __restrict__ x, float* __restrict__ lo, long long n) {
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  const long long n4 = (reinterpret_cast<uintptr_t>(x) & 15u) == 0 && (reinterpret_cast<uintptr_t>(lo) & 15u) == 0
                           ? n / 4
                           : 0;
  auto one = [](float v) { return to_tf32(v - __uint_as_float(__float_as_uint(v) & 0xffffe000u)); };
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n4; i += stride) {
    const float4 v = reinterpret_cast<const float4*>(x)[i];
    reinterpret_cast<float4*>(lo)[i] = make_float4(one(v.x), one(v.y), one(v.z), one(v.w));
  }
  for (long long i = 4 * n4 + blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n; i += stride)
    lo[i] = one(x[i]);
}

// Elements an operand of `rows` x `cols` with leading dimension `ld` spans.
long long footprint(long long rows, long long cols, long long ld) {
  return rows == 0 || cols == 0 ? 0 : (rows - 1) * ld + cols;
}

}  // namespace

void split_tf32(const float* x, float* hi, float* lo, long long n, cudaStream_t s) {
  if (n <= 0) return;
  const int threads = 256;
  long long blocks = (n + threads - 1) / threads;
  if (blocks > 148 * 32) blocks = 148 * 32;
  split_tf32_kernel<<<static_cast<int>(blocks), threads, 0, s>>>(x, hi, lo, n);
}

void split_lo_tf32(const float* x, float* lo, long long n, cudaStream_t s) {
  if (n <= 0) return;
  const int threads = 256;
  long long blocks = (n / 4 + threads - 1) / threads;
  if (blocks < 1) blocks = 1;
  if (blocks > 148 * 16) blocks = 148 * 16;
  split_lo_kernel<<<static_cast<int>(blocks), threads, 0, s>>>(x, lo, n);
}

namespace {

long long round4(long long n) { return (n + 3) & ~3ll; }

// K per tensor-memory accumulation in 3xTF32 (a multiple of 4, so that every
// chunk's first element stays 16-byte aligned for the tensor maps).
constexpr int kChunkK = 256;

}  // namespace

namespace {

// One product as one launch per K chunk of kChunkK (the shapes the CTA-pair
// kernel does not take): each launch accumulates one chunk from zero in tensor
// memory and its epilogue adds the result to the sum so far (R = C) in f32 on
// the CUDA cores, with round-to-nearest.
int gemm_3xtf32_chunked(int M, int N, int K, GemmOperand A, GemmOperand B, float* C, long long ldc,
                        const float* R, long long ldr, int* d_err, cudaStream_t stream) {
  if (M == 0 || N == 0 || K == 0) return gemm_tf32(M, N, K, A, B, C, ldc, R, ldr, d_err, stream);
  const long long na = A.mn_major ? footprint(K, M, A.ld) : footprint(M, K, A.ld);
  const long long nb = B.mn_major ? footprint(K, N, B.ld) : footprint(N, K, B.ld);
  const long long pa = round4(na), pb = round4(nb);
  float* ws = static_cast<float*>(device_scratch(static_cast<size_t>(2 * pa + 2 * pb) * sizeof(float), stream));
  float *a_hi = ws, *a_lo = ws + pa, *b_hi = ws + 2 * pa, *b_lo = ws + 2 * pa + pb;
  split_tf32(A.ptr, a_hi, a_lo, na, stream);
  split_tf32(B.ptr, b_hi, b_lo, nb, stream);
  int rc = 0;
  for (int k0 = 0; k0 < K && rc == 0; k0 += kChunkK) {
    const int kc = K - k0 < kChunkK ? K - k0 : kChunkK;
    auto at = [&](const float* base, const GemmOperand& op) {  // the operand from K index k0 on
      return op.mn_major ? base + static_cast<long long>(k0) * op.ld : base + k0;
    };
    GemmOperand Ah{at(a_hi, A), A.ld, A.mn_major}, Al{at(a_lo, A), A.ld, A.mn_major};
    GemmOperand Bh{at(b_hi, B), B.ld, B.mn_major}, Bl{at(b_lo, B), B.ld, B.mn_major};
    // Small terms first, then the large one, so the small ones are not rounded
    // away against a large partial sum before they are combined (one
    // accumulator over the three K ranges when the shape runs on CTA pairs).
    const GemmSegment terms[3] = {{Al, Bh, kc}, {Ah, Bl, kc}, {Ah, Bh, kc}};
    rc = gemm_tf32_sum(M, N, terms, 3, C, ldc, k0 == 0 ? R : C, k0 == 0 ? ldr : ldc, d_err, stream);
  }
  return rc;
}

}  // namespace

// The CTA-pair path splits only lo: hi is the operand itself, whose low 13
// mantissa bits the tensor core does not read (split_lo_kernel). The tensor
// core's f32 accumulation loses a little on every step, in the same
// direction, so its error grows linearly with the number of products summed in
// one accumulator (measured against float64: 4.8e-6 relative at K = 2048,
// 1.9e-5 at K = 8192 in one accumulation, where f32 on the CUDA cores stays at
// 0.8-1.6e-6). Both paths therefore sum short accumulations in f32 with
// round-to-nearest: the CTA-pair kernel every 64 of K (24 UMMAs) in registers,
// the chunked path every kChunkK of K through C.
X3LoCache::~X3LoCache() {
  for (Slot& s : slot)
    if (s.lo) cudaFree(s.lo);
}

namespace {

// The lo copy of `src` (n floats) from the cache, made when the cache does not
// hold it. Slots of this call (stamp) are never taken for another operand of
// it; otherwise the least recently used slot is, its buffer regrown in stream
// order when too small. Null when an allocation fails.
float* cached_lo(X3LoCache& c, const float* src, long long n, uint64_t stamp, cudaStream_t stream) {
  for (X3LoCache::Slot& s : c.slot)
    if (s.src == src && s.n == n) {
      s.stamp = stamp;
      return s.lo;
    }
  X3LoCache::Slot* v = nullptr;
  for (X3LoCache::Slot& s : c.slot)
    if (s.stamp != stamp && (!v || s.stamp < v->stamp)) v = &s;
  if (!v) return nullptr;
  if (v->cap < n) {
    if (v->lo && cudaFreeAsync(v->lo, stream) != cudaSuccess) return nullptr;
    v->lo = nullptr;
    v->cap = 0;
    void* p = nullptr;
    if (cudaMallocAsync(&p, static_cast<size_t>(round4(n)) * sizeof(float), stream) != cudaSuccess) return nullptr;
    v->lo = static_cast<float*>(p);
    v->cap = round4(n);
  }
  v->src = src;
  v->n = n;
  v->stamp = stamp;
  split_lo_tf32(src, v->lo, n, stream);
  return v->lo;
}

}  // namespace

int gemm_3xtf32_sum(int M, int N, const GemmSegment* segs, int nseg, float* C, long long ldc, const float* R,
                    long long ldr, int* d_err, cudaStream_t stream, X3LoCache* cache, bool keep) {
  if (cache && !keep)
    for (X3LoCache::Slot& s : cache->slot) s.src = nullptr;
  if (nseg < 1 || !segs) return kGemmBadArgument;
  GemmSegment live[3];
  int n_live = 0, n_k = 0;
  bool same = true;
  for (int g = 0; g < nseg; ++g) {
    if (segs[g].K < 0) return kGemmBadArgument;
    if (segs[g].K == 0) continue;
    if (n_live == 3) {
      same = false;
      break;
    }
    live[n_live] = segs[g];
    same = same && segs[g].a.mn_major == live[0].a.mn_major && segs[g].b.mn_major == live[0].b.mn_major;
    n_k += (segs[g].K + 31) / 32;
    ++n_live;
  }
  if (n_live == 0 || M == 0 || N == 0) return gemm_tf32_sum(M, N, segs, nseg, C, ldc, R, ldr, d_err, stream);
  if (same && gemm_3xtf32_pair_suits(M, N, n_k)) {
    // hi: the operands themselves (the tensor core reads their TF32 bits);
    // lo: what those bits leave out, rounded to TF32 (split_lo_tf32), from the
    // cache when one is given, else in the scratch arena
    const float* src[6];
    long long n[6], total = 0;
    bool kept[6];
    for (int g = 0; g < n_live; ++g) {
      const GemmSegment& s = live[g];
      if (!s.a.ptr || !s.b.ptr) return kGemmBadArgument;
      src[2 * g] = s.a.ptr;
      src[2 * g + 1] = s.b.ptr;
      n[2 * g] = s.a.mn_major ? footprint(s.K, M, s.a.ld) : footprint(M, s.K, s.a.ld);
      n[2 * g + 1] = s.b.mn_major ? footprint(s.K, N, s.b.ld) : footprint(N, s.K, s.b.ld);
    }
    for (int o = 0; o < 2 * n_live; ++o) {
      kept[o] = cache && n[o] <= X3LoCache::kMaxFloats;
      if (!kept[o]) total += round4(n[o]);
    }
    float* ws = total ? static_cast<float*>(device_scratch(static_cast<size_t>(total) * sizeof(float), stream))
                      : nullptr;
    const uint64_t stamp = cache ? ++cache->clock : 0;
    float* lo_of[6];
    for (int o = 0; o < 2 * n_live; ++o) {
      if (kept[o]) {
        lo_of[o] = cached_lo(*cache, src[o], n[o], stamp, stream);
        if (!lo_of[o]) return kGemmLaunch;
      } else {
        lo_of[o] = ws;
        ws += round4(n[o]);
        split_lo_tf32(src[o], lo_of[o], n[o], stream);
      }
    }
    GemmSegment hi[3], lo[3];
    for (int g = 0; g < n_live; ++g) {
      const GemmSegment& s = live[g];
      hi[g] = s;
      lo[g] = {{lo_of[2 * g], s.a.ld, s.a.mn_major}, {lo_of[2 * g + 1], s.b.ld, s.b.mn_major}, s.K};
    }
    return gemm_3xtf32_pair_sum(M, N, hi, lo, n_live, C, ldc, R, ldr, d_err, stream);
  }
  int rc = 0;
  bool first = true;
  for (int g = 0; g < nseg && rc == 0; ++g) {
    if (segs[g].K == 0) continue;
    rc = gemm_3xtf32_chunked(M, N, segs[g].K, segs[g].a, segs[g].b, C, ldc, first ? R : C, first ? ldr : ldc,
                             d_err, stream);
    first = false;
  }
  return rc;
}

int gemm_3xtf32(int M, int N, int K, GemmOperand A, GemmOperand B, float* C, long long ldc,
                const float* R, long long ldr, int* d_err, cudaStream_t stream) {
  if (K < 0) return kGemmBadArgument;
  const GemmSegment seg{A, B, K};
  return gemm_3xtf32_sum(M, N, &seg, 1, C, ldc, R, ldr, d_err, stream);
}

}  // namespace mm
