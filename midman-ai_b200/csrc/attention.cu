// Causal grouped-query flash attention (forward and backward), tiled 64 x 64 in
// shared memory with FP32 FMA micro-tiles. Scores never reach HBM: the forward
// keeps a running max/sum per query row (online softmax) and saves only the
// row's log-sum-exp; the backward recomputes P from it. Masked scores are
// skipped entirely, which equals the reference's -1e9 additive mask
// (attention.rs:24-27): exp(-1e9 - max) is exactly 0 in f32.
//
// Thread layout (256 threads): ty = tid / 16 owns 4 rows of a 64-row tile,
// tx = tid % 16 owns 4 score columns, or head dimensions tx, tx+16, ... of an
// output row. Grouped-query heads are addressed by index (h / group), so K and
// V are never expanded (attention.rs:59-65 copies them).
#include <cuda_runtime.h>

#include <cmath>
#include <stdexcept>
#include <string>

#include "attention.h"

namespace mm {

namespace {

constexpr int TILE = 64;
constexpr int PAD = 4;
constexpr int THREADS = 256;

void check(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

// Loads a 64-row tile of a token-major head slice into shared memory, either
// row-major [64][HD + PAD] or transposed [HD][64 + PAD]; rows past T are zero.
template <int HD, bool TRANSPOSED>
__device__ __forceinline__ void load_tile(float* dst, const float* src, long long ld, int row0, int T, int hd) {
  for (int idx = threadIdx.x; idx < TILE * HD; idx += THREADS) {
    const int r = idx / HD, d = idx % HD;
    float val = 0.0f;
    if (d < hd && row0 + r < T) val = src[static_cast<long long>(row0 + r) * ld + d];
    if (TRANSPOSED)
      dst[d * (TILE + PAD) + r] = val;
    else
      dst[r * (HD + PAD) + d] = val;
  }
}

template <int HD>
__global__ void __launch_bounds__(THREADS) attn_fwd_kernel(AttnShape s, const float* __restrict__ q,
                                                           const float* __restrict__ k, const float* __restrict__ v,
                                                           float* __restrict__ o, float* __restrict__ lse) {
  extern __shared__ float smem[];
  float* Qt = smem;                          // [HD][TILE + PAD]
  float* Kt = Qt + HD * (TILE + PAD);        // [HD][TILE + PAD]
  float* Vs = Kt + HD * (TILE + PAD);        // [TILE][HD + PAD]
  float* Ps = Vs + TILE * (HD + PAD);        // [TILE][TILE + PAD]
  constexpr int DJ = HD / 16;
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (s.H / s.Hkv);
  const int ty = threadIdx.x / 16, tx = threadIdx.x % 16;
  const int q0 = qt * TILE;
  const long long base = static_cast<long long>(b) * s.T;
  load_tile<HD, true>(Qt, q + base * s.ldq + static_cast<long long>(h) * s.hd, s.ldq, q0, s.T, s.hd);
  float m[4], l[4], acc[4][DJ];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.0f;
#pragma unroll
    for (int j = 0; j < DJ; ++j) acc[i][j] = 0.0f;
  }
  for (int kt = 0; kt <= qt; ++kt) {
    const int k0 = kt * TILE;
    __syncthreads();
    load_tile<HD, true>(Kt, k + base * s.ldk + static_cast<long long>(hk) * s.hd, s.ldk, k0, s.T, s.hd);
    load_tile<HD, false>(Vs, v + base * s.ldv + static_cast<long long>(hk) * s.hd, s.ldv, k0, s.T, s.hd);
    __syncthreads();
    float sc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) sc[i][j] = 0.0f;
    for (int d = 0; d < s.hd; ++d) {
      const float4 a = *reinterpret_cast<const float4*>(&Qt[d * (TILE + PAD) + 4 * ty]);
      const float4 c = *reinterpret_cast<const float4*>(&Kt[d * (TILE + PAD) + 4 * tx]);
      const float av[4] = {a.x, a.y, a.z, a.w}, cv[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) sc[i][j] += av[i] * cv[j];
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int row = q0 + 4 * ty + i;
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int col = k0 + 4 * tx + j;
        sc[i][j] = (col <= row && col < s.T && row < s.T) ? sc[i][j] * s.scale : -INFINITY;
        mx = fmaxf(mx, sc[i][j]);
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float mnew = fmaxf(m[i], mx);
      float rs = 0.0f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float p = mnew == -INFINITY ? 0.0f : expf(sc[i][j] - mnew);
        sc[i][j] = p;
        rs += p;
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) rs += __shfl_xor_sync(0xffffffffu, rs, off);
      const float alpha = (m[i] == -INFINITY) ? 0.0f : expf(m[i] - mnew);
      l[i] = l[i] * alpha + rs;
      m[i] = mnew;
#pragma unroll
      for (int j = 0; j < DJ; ++j) acc[i][j] *= alpha;
      *reinterpret_cast<float4*>(&Ps[(4 * ty + i) * (TILE + PAD) + 4 * tx]) =
          make_float4(sc[i][0], sc[i][1], sc[i][2], sc[i][3]);
    }
    __syncthreads();
    const int kmax = min(TILE, s.T - k0);
    for (int c = 0; c < kmax; ++c) {
      float pv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) pv[i] = Ps[(4 * ty + i) * (TILE + PAD) + c];
#pragma unroll
      for (int j = 0; j < DJ; ++j) {
        const float vv = Vs[c * (HD + PAD) + tx + 16 * j];
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[i][j] += pv[i] * vv;
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int row = q0 + 4 * ty + i;
    if (row >= s.T) continue;
    const float inv = 1.0f / l[i];
    float* orow = o + (base + row) * s.ldo + static_cast<long long>(h) * s.hd;
#pragma unroll
    for (int j = 0; j < DJ; ++j) {
      const int d = tx + 16 * j;
      if (d < s.hd) orow[d] = acc[i][j] * inv;
    }
    if (tx == 0) lse[(static_cast<long long>(b) * s.H + h) * s.T + row] = m[i] + logf(l[i]);
  }
}

// delta[b, h, t] = sum_d do[t, d] * o[t, d] (one warp per row).
__global__ void attn_delta_kernel(AttnShape s, const float* __restrict__ o, const float* __restrict__ dout,
                                  long long lddo, float* __restrict__ delta) {
  const long long warp = (blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x) / 32;
  const int lane = threadIdx.x & 31;
  const long long rows = static_cast<long long>(s.B) * s.H * s.T;
  if (warp >= rows) return;
  const int t = static_cast<int>(warp % s.T);
  const int h = static_cast<int>((warp / s.T) % s.H);
  const int b = static_cast<int>(warp / (static_cast<long long>(s.T) * s.H));
  const long long tok = static_cast<long long>(b) * s.T + t;
  const float* orow = o + tok * s.ldo + static_cast<long long>(h) * s.hd;
  const float* drow = dout + tok * lddo + static_cast<long long>(h) * s.hd;
  float acc = 0.0f;
  for (int d = lane; d < s.hd; d += 32) acc += orow[d] * drow[d];
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (lane == 0) delta[warp] = acc;
}


// Scores and dP for one 64 x 64 tile: rows 4ty+i of Qs/dOs against columns
// 4tx+j of Kt/Vt. Then P = exp(S*scale - lse) under the causal mask and
// dS = P * (dP - delta) (the softmax backward, ops_reduce.rs:131-142).
template <int HD>
__device__ __forceinline__ void tile_p_ds(const AttnShape& s, const float* Qs, const float* dOs, const float* Kt,
                                          const float* Vt, const float* lse_s, const float* del_s, int q0, int k0,
                                          int ty, int tx, float (&p)[4][4], float (&ds)[4][4]) {
  float sc[4][4], dp[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) sc[i][j] = dp[i][j] = 0.0f;
  for (int d = 0; d < s.hd; ++d) {
    const float4 kb = *reinterpret_cast<const float4*>(&Kt[d * (TILE + PAD) + 4 * tx]);
    const float4 vb = *reinterpret_cast<const float4*>(&Vt[d * (TILE + PAD) + 4 * tx]);
    const float kv[4] = {kb.x, kb.y, kb.z, kb.w}, vv[4] = {vb.x, vb.y, vb.z, vb.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float qa = Qs[(4 * ty + i) * (HD + PAD) + d];
      const float da = dOs[(4 * ty + i) * (HD + PAD) + d];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        sc[i][j] += qa * kv[j];
        dp[i][j] += da * vv[j];
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = 4 * ty + i, row = q0 + r;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int col = k0 + 4 * tx + j;
      const bool live = col <= row && row < s.T && col < s.T;
      p[i][j] = live ? expf(sc[i][j] * s.scale - lse_s[r]) : 0.0f;
      ds[i][j] = p[i][j] * (dp[i][j] - del_s[r]);
    }
  }
}

template <int HD>
__global__ void __launch_bounds__(THREADS) attn_bwd_kv_kernel(AttnShape s, const float* __restrict__ q,
                                                              const float* __restrict__ k, const float* __restrict__ v,
                                                              const float* __restrict__ dout, long long lddo,
                                                              const float* __restrict__ lse,
                                                              const float* __restrict__ delta, float* __restrict__ dk,
                                                              float* __restrict__ dv) {
  extern __shared__ float smem[];
  float* Qs = smem;                        // [TILE][HD + PAD]
  float* dOs = Qs + TILE * (HD + PAD);     // [TILE][HD + PAD]
  float* Kt = dOs + TILE * (HD + PAD);     // [HD][TILE + PAD]
  float* Vt = Kt + HD * (TILE + PAD);      // [HD][TILE + PAD]
  float* Ps = Vt + HD * (TILE + PAD);      // [TILE][TILE + PAD]
  float* dSs = Ps + TILE * (TILE + PAD);   // [TILE][TILE + PAD]
  float* lse_s = dSs + TILE * (TILE + PAD);
  float* del_s = lse_s + TILE;
  constexpr int DJ = HD / 16;
  const int kt = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
  const int group = s.H / s.Hkv;
  const int ty = threadIdx.x / 16, tx = threadIdx.x % 16;
  const int k0 = kt * TILE;
  const long long base = static_cast<long long>(b) * s.T;
  load_tile<HD, true>(Kt, k + base * s.ldk + static_cast<long long>(hk) * s.hd, s.ldk, k0, s.T, s.hd);
  load_tile<HD, true>(Vt, v + base * s.ldv + static_cast<long long>(hk) * s.hd, s.ldv, k0, s.T, s.hd);
  float dK[4][DJ], dV[4][DJ];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < DJ; ++j) dK[i][j] = dV[i][j] = 0.0f;
  const int n_tiles = (s.T + TILE - 1) / TILE;
  for (int hh = 0; hh < group; ++hh) {
    const int h = hk * group + hh;
    for (int qt = kt; qt < n_tiles; ++qt) {
      const int q0 = qt * TILE;
      __syncthreads();
      load_tile<HD, false>(Qs, q + base * s.ldq + static_cast<long long>(h) * s.hd, s.ldq, q0, s.T, s.hd);
      load_tile<HD, false>(dOs, dout + base * lddo + static_cast<long long>(h) * s.hd, lddo, q0, s.T, s.hd);
      if (threadIdx.x < TILE) {
        const int row = q0 + threadIdx.x;
        const long long li = (static_cast<long long>(b) * s.H + h) * s.T + row;
        lse_s[threadIdx.x] = row < s.T ? lse[li] : 0.0f;
        del_s[threadIdx.x] = row < s.T ? delta[li] : 0.0f;
      }
      __syncthreads();
      float p[4][4], ds[4][4];
      tile_p_ds<HD>(s, Qs, dOs, Kt, Vt, lse_s, del_s, q0, k0, ty, tx, p, ds);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        *reinterpret_cast<float4*>(&Ps[(4 * ty + i) * (TILE + PAD) + 4 * tx]) =
            make_float4(p[i][0], p[i][1], p[i][2], p[i][3]);
        *reinterpret_cast<float4*>(&dSs[(4 * ty + i) * (TILE + PAD) + 4 * tx]) =
            make_float4(ds[i][0], ds[i][1], ds[i][2], ds[i][3]);
      }
      __syncthreads();
      const int rmax = min(TILE, s.T - q0);
      for (int r = 0; r < rmax; ++r) {
        const float4 p4 = *reinterpret_cast<const float4*>(&Ps[r * (TILE + PAD) + 4 * ty]);
        const float4 d4 = *reinterpret_cast<const float4*>(&dSs[r * (TILE + PAD) + 4 * ty]);
        const float pv[4] = {p4.x, p4.y, p4.z, p4.w}, dv4[4] = {d4.x, d4.y, d4.z, d4.w};
#pragma unroll
        for (int j = 0; j < DJ; ++j) {
          const float dov = dOs[r * (HD + PAD) + tx + 16 * j];
          const float qv = Qs[r * (HD + PAD) + tx + 16 * j];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            dV[i][j] += pv[i] * dov;
            dK[i][j] += dv4[i] * qv;
          }
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int key = k0 + 4 * ty + i;
    if (key >= s.T) continue;
    float* dkr = dk + (base + key) * s.ldk + static_cast<long long>(hk) * s.hd;
    float* dvr = dv + (base + key) * s.ldv + static_cast<long long>(hk) * s.hd;
#pragma unroll
    for (int j = 0; j < DJ; ++j) {
      const int d = tx + 16 * j;
      if (d < s.hd) {
        dkr[d] = dK[i][j] * s.scale;
        dvr[d] = dV[i][j];
      }
    }
  }
}

template <int HD>
__global__ void __launch_bounds__(THREADS) attn_bwd_q_kernel(AttnShape s, const float* __restrict__ q,
                                                             const float* __restrict__ k, const float* __restrict__ v,
                                                             const float* __restrict__ dout, long long lddo,
                                                             const float* __restrict__ lse,
                                                             const float* __restrict__ delta, float* __restrict__ dq) {
  extern __shared__ float smem[];
  float* Qs = smem;                        // [TILE][HD + PAD]
  float* dOs = Qs + TILE * (HD + PAD);     // [TILE][HD + PAD]
  float* Kt = dOs + TILE * (HD + PAD);     // [HD][TILE + PAD]
  float* Ks = Kt + HD * (TILE + PAD);      // [TILE][HD + PAD]
  float* Vt = Ks + TILE * (HD + PAD);      // [HD][TILE + PAD]
  float* dSs = Vt + HD * (TILE + PAD);     // [TILE][TILE + PAD]
  float* lse_s = dSs + TILE * (TILE + PAD);
  float* del_s = lse_s + TILE;
  constexpr int DJ = HD / 16;
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (s.H / s.Hkv);
  const int ty = threadIdx.x / 16, tx = threadIdx.x % 16;
  const int q0 = qt * TILE;
  const long long base = static_cast<long long>(b) * s.T;
  load_tile<HD, false>(Qs, q + base * s.ldq + static_cast<long long>(h) * s.hd, s.ldq, q0, s.T, s.hd);
  load_tile<HD, false>(dOs, dout + base * lddo + static_cast<long long>(h) * s.hd, lddo, q0, s.T, s.hd);
  if (threadIdx.x < TILE) {
    const int row = q0 + threadIdx.x;
    const long long li = (static_cast<long long>(b) * s.H + h) * s.T + row;
    lse_s[threadIdx.x] = row < s.T ? lse[li] : 0.0f;
    del_s[threadIdx.x] = row < s.T ? delta[li] : 0.0f;
  }
  float dQ[4][DJ];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < DJ; ++j) dQ[i][j] = 0.0f;
  for (int kt = 0; kt <= qt; ++kt) {
    const int k0 = kt * TILE;
    __syncthreads();
    const float* kb = k + base * s.ldk + static_cast<long long>(hk) * s.hd;
    load_tile<HD, true>(Kt, kb, s.ldk, k0, s.T, s.hd);
    load_tile<HD, false>(Ks, kb, s.ldk, k0, s.T, s.hd);
    load_tile<HD, true>(Vt, v + base * s.ldv + static_cast<long long>(hk) * s.hd, s.ldv, k0, s.T, s.hd);
    __syncthreads();
    float p[4][4], ds[4][4];
    tile_p_ds<HD>(s, Qs, dOs, Kt, Vt, lse_s, del_s, q0, k0, ty, tx, p, ds);
#pragma unroll
    for (int i = 0; i < 4; ++i)
      *reinterpret_cast<float4*>(&dSs[(4 * ty + i) * (TILE + PAD) + 4 * tx]) =
          make_float4(ds[i][0], ds[i][1], ds[i][2], ds[i][3]);
    __syncthreads();
    const int cmax = min(TILE, s.T - k0);
    for (int c = 0; c < cmax; ++c) {
      float dsv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) dsv[i] = dSs[(4 * ty + i) * (TILE + PAD) + c];
#pragma unroll
      for (int j = 0; j < DJ; ++j) {
        const float kv = Ks[c * (HD + PAD) + tx + 16 * j];
#pragma unroll
        for (int i = 0; i < 4; ++i) dQ[i][j] += dsv[i] * kv;
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int row = q0 + 4 * ty + i;
    if (row >= s.T) continue;
    float* dqr = dq + (base + row) * s.ldq + static_cast<long long>(h) * s.hd;
#pragma unroll
    for (int j = 0; j < DJ; ++j) {
      const int d = tx + 16 * j;
      if (d < s.hd) dqr[d] = dQ[i][j] * s.scale;
    }
  }
}

__global__ void attn_probs_kernel(AttnShape s, const float* __restrict__ q, const float* __restrict__ k,
                                  const float* __restrict__ lse, float* __restrict__ probs) {
  const long long total = static_cast<long long>(s.B) * s.H * s.T * s.T;
  for (long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int j = static_cast<int>(idx % s.T);
    const long long bhi = idx / s.T;
    const int i = static_cast<int>(bhi % s.T);
    const long long bh = bhi / s.T;
    const int h = static_cast<int>(bh % s.H);
    const int b = static_cast<int>(bh / s.H);
    float p = 0.0f;
    if (j <= i) {
      const int hk = h / (s.H / s.Hkv);
      const float* qr = q + (static_cast<long long>(b) * s.T + i) * s.ldq + static_cast<long long>(h) * s.hd;
      const float* kr = k + (static_cast<long long>(b) * s.T + j) * s.ldk + static_cast<long long>(hk) * s.hd;
      float acc = 0.0f;
      for (int d = 0; d < s.hd; ++d) acc += qr[d] * kr[d];
      p = expf(acc * s.scale - lse[bhi]);
    }
    probs[idx] = p;
  }
}

template <int HD>
size_t fwd_smem() { return sizeof(float) * (2 * HD * (TILE + PAD) + TILE * (HD + PAD) + TILE * (TILE + PAD)); }
template <int HD>
size_t kv_smem() {
  return sizeof(float) * (2 * TILE * (HD + PAD) + 2 * HD * (TILE + PAD) + 2 * TILE * (TILE + PAD) + 2 * TILE);
}
template <int HD>
size_t q_smem() {
  return sizeof(float) * (3 * TILE * (HD + PAD) + 2 * HD * (TILE + PAD) + TILE * (TILE + PAD) + 2 * TILE);
}

template <int HD>
void launch_fwd(const AttnShape& s, const float* q, const float* k, const float* v, float* o, float* lse,
                cudaStream_t st) {
  const size_t sm = fwd_smem<HD>();
  cudaFuncSetAttribute(attn_fwd_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(sm));
  dim3 grid((s.T + TILE - 1) / TILE, s.H, s.B);
  attn_fwd_kernel<HD><<<grid, THREADS, sm, st>>>(s, q, k, v, o, lse);
  check("attention_forward");
}

template <int HD>
void launch_bwd(const AttnShape& s, const float* q, const float* k, const float* v, const float* dout, long long lddo,
                const float* lse, const float* delta, float* dq, float* dk, float* dv, cudaStream_t st) {
  const size_t skv = kv_smem<HD>(), sq = q_smem<HD>();
  cudaFuncSetAttribute(attn_bwd_kv_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(skv));
  cudaFuncSetAttribute(attn_bwd_q_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(sq));
  const int tiles = (s.T + TILE - 1) / TILE;
  attn_bwd_kv_kernel<HD><<<dim3(tiles, s.Hkv, s.B), THREADS, skv, st>>>(s, q, k, v, dout, lddo, lse, delta, dk, dv);
  check("attention_backward(dk, dv)");
  attn_bwd_q_kernel<HD><<<dim3(tiles, s.H, s.B), THREADS, sq, st>>>(s, q, k, v, dout, lddo, lse, delta, dq);
  check("attention_backward(dq)");
}

void validate(const AttnShape& s) {
  if (s.B <= 0 || s.T <= 0 || s.H <= 0 || s.Hkv <= 0 || s.H % s.Hkv != 0 || s.hd <= 0 || s.hd > 128)
    throw std::runtime_error("attention: unsupported shape (head_dim must be 1..128, heads a multiple of kv heads)");
}

}  // namespace

void attention_forward(const AttnShape& s, const float* q, const float* k, const float* v, float* o, float* lse,
                       cudaStream_t stream) {
  validate(s);
  if (s.hd <= 16) launch_fwd<16>(s, q, k, v, o, lse, stream);
  else if (s.hd <= 32) launch_fwd<32>(s, q, k, v, o, lse, stream);
  else if (s.hd <= 64) launch_fwd<64>(s, q, k, v, o, lse, stream);
  else launch_fwd<128>(s, q, k, v, o, lse, stream);
}

void attention_backward(const AttnShape& s, const float* q, const float* k, const float* v, const float* o,
                        const float* lse, const float* dout, long long lddo, float* dq, float* dk, float* dv,
                        float* delta, cudaStream_t stream) {
  validate(s);
  attention_delta(s, o, dout, lddo, delta, stream);
  if (s.hd <= 16) launch_bwd<16>(s, q, k, v, dout, lddo, lse, delta, dq, dk, dv, stream);
  else if (s.hd <= 32) launch_bwd<32>(s, q, k, v, dout, lddo, lse, delta, dq, dk, dv, stream);
  else if (s.hd <= 64) launch_bwd<64>(s, q, k, v, dout, lddo, lse, delta, dq, dk, dv, stream);
  else launch_bwd<128>(s, q, k, v, dout, lddo, lse, delta, dq, dk, dv, stream);
}

void attention_delta(const AttnShape& s, const float* o, const float* dout, long long lddo, float* delta,
                     cudaStream_t stream) {
  const long long rows = static_cast<long long>(s.B) * s.H * s.T;
  attn_delta_kernel<<<static_cast<unsigned>((rows * 32 + 255) / 256), 256, 0, stream>>>(s, o, dout, lddo, delta);
  check("attention delta");
}

void attention_probs(const AttnShape& s, const float* q, const float* k, const float* lse, float* probs,
                     cudaStream_t stream) {
  validate(s);
  const long long total = static_cast<long long>(s.B) * s.H * s.T * s.T;
  long long blocks = (total + 255) / 256;
  if (blocks > 148 * 64) blocks = 148 * 64;
  attn_probs_kernel<<<static_cast<int>(blocks), 256, 0, stream>>>(s, q, k, lse, probs);
  check("attention_probs");
}

}  // namespace mm
