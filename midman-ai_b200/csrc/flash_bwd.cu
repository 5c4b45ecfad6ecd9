// Fused causal attention backward on the tensor cores (TF32, tcgen05 + TMEM).
//
// The backward of attention.rs:79-102 (the reference differentiates it through
// its autograd tape), split FA2-style into two kernels that never write a
// score-sized buffer:
//
//   flash_bwd_kv  one CTA per (128-key tile, batch, key/value head); loops over
//                 the group's query heads and the query blocks (32 queries) at
//                 or after the tile's first key. Per block, lanes = keys:
//                   S^T  = K Q^T          A = K (smem), B = Q (smem, K-major)
//                   dP^T = V dO^T         A = V (TMEM),  B = dO (smem, K-major)
//                   P = exp(S*scale - lse), dS = P (dP - delta) * scale  (softmax warps)
//                   dV  += P^T-rows dO    A = P  (TMEM), B = dO (smem, MN-major)
//                   dK  += dS^T-rows Q    A = dS (TMEM), B = Q  (smem, MN-major)
//                 dK and dV of the key/value head accumulate in TMEM over the
//                 whole group, so grouped-query heads need no reduction pass.
//   flash_bwd_q   one CTA per (128-query tile, batch, head); loops over key
//                 blocks (32 keys) up to the diagonal. Lanes = queries:
//                   S  = Q K^T            A = Q (smem),  B = K (smem, K-major)
//                   dP = dO V^T           A = dO (TMEM), B = V (smem, K-major)
//                   dS = P (dP - delta) * scale
//                   dQ += dS K            A = dS (TMEM), B = K (smem, MN-major)
//
// An fp32 [rows, hd] tile serves as a K-major operand (hd contracted) with the
// 16-byte-atom 128-byte swizzle and as an MN-major operand (hd the output
// dimension) only with the 32-byte-atom swizzle, so those tiles are loaded
// twice, once per layout. delta = rowsum(dO * O) comes from attention_delta.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <stdexcept>
#include <string>

#include "attention.h"
#include "ptx.cuh"
#include "tma.h"

namespace mm {

namespace {

constexpr int TILE = 128;  // lanes: keys (kv kernel) or queries (q kernel)
constexpr int BLK = 32;    // streamed queries (kv kernel) or keys (q kernel) per step
constexpr int BTHREADS = 320;  // producer, UMMA issuer, two softmax warpgroups
constexpr float kLog2e = 1.4426950408889634f;

struct BwdParams {
  int T, H, Hkv, G, n_tiles, BHx;  // BHx = B * heads the grid runs over
  long long ld_in;                 // row stride of the operand loaded into TMEM (v or dout)
  long long ld_out;                // row stride of the outputs
  long long ld_out2;               // dv (kv kernel)
  const float* tm_src;             // that operand
  const float* lse;
  const float* delta;
  float* out;   // dk (kv kernel) or dq (q kernel)
  float* out2;  // dv (kv kernel)
  float scale, scale_log2;
  int* err;
};

template <int HD>
struct BwdCfg {
  static constexpr int TILE_BYTES = TILE * HD * 4;  // resident K (kv) or Q (q)
  static constexpr int BLK_BYTES = BLK * HD * 4;    // one streamed tile
  // kv kernel streams Q, dO (K-major) and Q, dO (MN-major); q kernel K, V (K-major) and K (MN-major)
  static constexpr int KV_STAGE = 4 * BLK_BYTES;
  static constexpr int Q_STAGE = 3 * BLK_BYTES;
  static constexpr int KV_STAGES_FIT = (210 * 1024 - TILE_BYTES) / KV_STAGE;
  static constexpr int Q_STAGES_FIT = (210 * 1024 - TILE_BYTES) / Q_STAGE;
  static constexpr int KV_STAGES = KV_STAGES_FIT > 4 ? 4 : KV_STAGES_FIT;
  static constexpr int Q_STAGES = Q_STAGES_FIT > 4 ? 4 : Q_STAGES_FIT;
  static constexpr int KV_SMEM = TILE_BYTES + KV_STAGES * KV_STAGE + 1024 + 256;
  static constexpr int Q_SMEM = TILE_BYTES + Q_STAGES * Q_STAGE + 1024 + 256;
  // TMEM: 2 x (S/P, dP/dS) buffers of BLK columns, then the TMEM-resident
  // operand and the accumulators, hd columns each
  static constexpr uint32_t BUF_COLS = 4 * BLK;      // 128
  static constexpr uint32_t OPND_COL = BUF_COLS;     // V (kv) or dO (q)
  static constexpr uint32_t ACC_COL = BUF_COLS + HD; // dV (kv) or dQ (q)
  static constexpr uint32_t ACC2_COL = ACC_COL + HD; // dK (kv)
  static constexpr uint32_t TMEM_COLS = 512;
  static_assert(KV_STAGES >= 2 && Q_STAGES >= 2, "backward needs two stages");
  static_assert(ACC2_COL + HD <= TMEM_COLS, "TMEM budget");
};

__device__ __forceinline__ uint32_t s_col_of(int bb, int blk) { return bb * 2 * blk; }         // S / P
__device__ __forceinline__ uint32_t dp_col_of(int bb, int blk) { return bb * 2 * blk + blk; }  // dP / dS
__device__ __forceinline__ uint32_t s_col(int bb) { return s_col_of(bb, BLK); }
__device__ __forceinline__ uint32_t dp_col(int bb) { return dp_col_of(bb, BLK); }

// Barrier block shared by both kernels (offsets in 8-byte slots).
template <int STAGES>
struct Bars {
  uint32_t base;
  __device__ uint32_t tile_full() const { return base; }
  __device__ uint32_t full(int s) const { return base + 8u * (1 + s); }
  __device__ uint32_t empty(int s) const { return base + 8u * (1 + STAGES + s); }
  __device__ uint32_t s_full(int bb) const { return base + 8u * (1 + 2 * STAGES + bb); }
  __device__ uint32_t p_full(int bb) const { return base + 8u * (3 + 2 * STAGES + bb); }
  __device__ uint32_t s_free(int bb) const { return base + 8u * (5 + 2 * STAGES + bb); }
  __device__ uint32_t opnd_ready() const { return base + 8u * (7 + 2 * STAGES); }
  __device__ uint32_t acc_done() const { return base + 8u * (8 + 2 * STAGES); }
  __device__ uint32_t slot() const { return base + 8u * (9 + 2 * STAGES); }
  __device__ void init() const {
    mbar_init(tile_full(), 1);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full(s), 1);
      mbar_init(empty(s), 1);
    }
    for (int bb = 0; bb < 2; ++bb) {
      mbar_init(s_full(bb), 1);
      mbar_init(p_full(bb), 4);
      mbar_init(s_free(bb), 1);
    }
    mbar_init(opnd_ready(), 8);  // every softmax warp
    mbar_init(acc_done(), 1);
  }
};

// Byte offset of contraction step kk (8 tf32) in a K-major tile of `rows` rows
// stored as 128-byte chunks of 32 elements (chunk stride rows * 128 bytes).
__host__ __device__ constexpr uint32_t kchunk_off(int rows, int kk) {
  return static_cast<uint32_t>((kk / 4) * (rows * 128) + (kk % 4) * 32);
}

// K-major descriptor of contraction step kk (8 tf32) in a tile of `rows` rows
// stored as 128-byte chunks of 32 elements (chunk stride rows * 128 bytes).
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t tile, int rows, int kk) {
  return smem_desc(tile + (kk / 4) * (rows * 128) + (kk % 4) * 32, 16, 1024, kLayoutSw128);
}
// MN-major descriptor of contraction step kk (8 rows) in a BLK-row tile stored
// as 32-column blocks of BLK rows (block stride BLK * 128 bytes).
__device__ __forceinline__ uint64_t mnmajor_desc(uint32_t tile, int kk) {
  return smem_desc(tile + kk * 1024, BLK * 128, 512, kLayoutSw128Base32);
}

// Copies 32-column chunks c0, c0 + 2, ... of a row (HD floats at src, or zeros
// when !valid) into the same TMEM columns of this thread's lane.
template <int HD>
__device__ __forceinline__ void row_to_tmem(const float* src, bool valid, uint32_t taddr, int c0) {
#pragma unroll 1
  for (int c = c0; c < HD / 32; c += 2) {
    uint32_t r[32];
#pragma unroll
    for (int i = 0; i < 32; i += 4) {
      float4 v = valid ? *reinterpret_cast<const float4*>(src + c * 32 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
      r[i] = __float_as_uint(v.x);
      r[i + 1] = __float_as_uint(v.y);
      r[i + 2] = __float_as_uint(v.z);
      r[i + 3] = __float_as_uint(v.w);
    }
    tmem_st_32x32b_x32(taddr + c * 32, r);
  }
}

// Writes 32-column chunks c0, c0 + step, ... of this thread's TMEM lane, times
// `mul`, to the same columns of dst.
template <int HD>
__device__ __forceinline__ void tmem_to_row(uint32_t taddr, float* dst, bool valid, float mul, int c0 = 0,
                                            int step = 1) {
#pragma unroll 1
  for (int c = c0; c < HD / 32; c += step) {
    uint32_t r[32];
    tmem_ld_32x32b_x32(taddr + c * 32, r);
    if (valid) {
#pragma unroll
      for (int i = 0; i < 32; i += 4)
        *reinterpret_cast<float4*>(dst + c * 32 + i) =
            make_float4(__uint_as_float(r[i]) * mul, __uint_as_float(r[i + 1]) * mul,
                        __uint_as_float(r[i + 2]) * mul, __uint_as_float(r[i + 3]) * mul);
    }
  }
}

// Loads 32-column chunks c0, c0 + 2, ... of rows row_first .. row_first + 31 of
// src (`ld` apart; rows at or past n_rows read as 0) into this warp's 32 TMEM
// lanes through the warp's 32 x 16 staging tile `wst`, so that each load
// instruction reads eight whole 64-byte row segments.
template <int HD>
__device__ __forceinline__ void rows_to_tmem(const float* src, long long ld, int row_first, int n_rows,
                                             uint32_t taddr, float4* wst, int c0) {
  const int lane = threadIdx.x % 32, sub = lane & 3, rsub = lane >> 2;
#pragma unroll 1
  for (int c = c0; c < HD / 32; c += 2) {
    uint32_t r[32];
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      float4 v[4];
#pragma unroll
      for (int it = 0; it < 4; ++it) {
        const int rr = it * 8 + rsub;
        v[it] = row_first + rr < n_rows
                    ? *reinterpret_cast<const float4*>(src + static_cast<long long>(row_first + rr) * ld + c * 32 +
                                                       half * 16 + sub * 4)
                    : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int it = 0; it < 4; ++it) {
        const int rr = it * 8 + rsub;
        wst[rr * 4 + (sub ^ (rr & 3))] = v[it];
      }
      __syncwarp();
#pragma unroll
      for (int gr = 0; gr < 4; ++gr) {
        const float4 w = wst[lane * 4 + (gr ^ (lane & 3))];
        const int i = half * 16 + gr * 4;
        r[i] = __float_as_uint(w.x);
        r[i + 1] = __float_as_uint(w.y);
        r[i + 2] = __float_as_uint(w.z);
        r[i + 3] = __float_as_uint(w.w);
      }
      __syncwarp();
    }
    tmem_st_32x32b_x32(taddr + c * 32, r);
  }
}

// Writes 32-column chunks c0, c0 + step, ... of this warp's 32 TMEM lanes to
// rows row_first .. row_first + 31 of dst (`ld` apart; rows at or past n_rows
// are skipped) through the warp's 32 x 16 staging tile `wst` (4-float granules
// XOR-swizzled by row), so that each store instruction writes eight whole
// 64-byte row segments.
template <int HD>
__device__ __forceinline__ void tmem_to_rows(uint32_t taddr, float* dst, long long ld, int row_first, int n_rows,
                                             float4* wst, int c0 = 0, int step = 1) {
  const int lane = threadIdx.x % 32, sub = lane & 3, rsub = lane >> 2;
#pragma unroll 1
  for (int c = c0; c < HD / 32; c += step) {
    uint32_t r[32];
    tmem_ld_32x32b_x32(taddr + c * 32, r);
#pragma unroll
    for (int half = 0; half < 2; ++half) {
#pragma unroll
      for (int gr = 0; gr < 4; ++gr) {
        const int i = half * 16 + gr * 4;
        wst[lane * 4 + (gr ^ (lane & 3))] = make_float4(__uint_as_float(r[i]), __uint_as_float(r[i + 1]),
                                                        __uint_as_float(r[i + 2]), __uint_as_float(r[i + 3]));
      }
      __syncwarp();
#pragma unroll
      for (int it = 0; it < 4; ++it) {
        const int rr = it * 8 + rsub;
        const float4 v = wst[rr * 4 + (sub ^ (rr & 3))];
        if (row_first + rr < n_rows)
          *reinterpret_cast<float4*>(dst + static_cast<long long>(row_first + rr) * ld + c * 32 + half * 16 + sub * 4) =
              v;
      }
      __syncwarp();
    }
  }
}

// out[i] = src[i] * mul for the first n_valid of 32 consecutive floats, 0 past them.
__device__ __forceinline__ void load32(const float* src, int n_valid, float mul, float (&out)[32]) {
  if (n_valid >= 32 && (reinterpret_cast<uintptr_t>(src) & 15u) == 0) {
#pragma unroll
    for (int i = 0; i < 32; i += 4) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(src + i));
      out[i] = v.x * mul;
      out[i + 1] = v.y * mul;
      out[i + 2] = v.z * mul;
      out[i + 3] = v.w * mul;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) out[i] = i < n_valid ? __ldg(src + i) * mul : 0.0f;
  }
}

// Shared-memory tail after the barriers: TMEM address slot and pipeline counters.
struct Tail {
  uint32_t tmem;
  int pad;
  int issued, consumed, tile_pending;
};

template <int STAGES, class B>
__device__ __forceinline__ void drain(const B& bars, Tail* tl, int* err) {
  if (tl->tile_pending) mbar_wait(bars.tile_full(), 0, err, kErrWaitDrain, 1000000000ull);
  for (int t = tl->consumed; t < tl->issued; ++t)
    if (!mbar_wait(bars.full(t % STAGES), (t / STAGES) & 1, err, kErrWaitDrain, 1000000000ull)) break;
}

// ------------------------------------------------------------------ dK, dV
template <int HD>
__global__ void __launch_bounds__(BTHREADS, 1)
    flash_bwd_kv_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmQk,
                        const __grid_constant__ CUtensorMap tmDOk, const __grid_constant__ CUtensorMap tmQm,
                        const __grid_constant__ CUtensorMap tmDOm, BwdParams p) {
  using Cfg = BwdCfg<HD>;
  constexpr int STAGES = Cfg::KV_STAGES;
  constexpr int BB = Cfg::BLK_BYTES;
  const int kt = static_cast<int>(blockIdx.x) / p.BHx;  // low key tiles see the most queries: first
  const int bhk = static_cast<int>(blockIdx.x) % p.BHx;
  const int b = bhk / p.Hkv, hk = bhk % p.Hkv;
  const int k0 = kt * TILE;
  const int row0 = b * p.T;
  const int n_q = (p.T - k0 + BLK - 1) / BLK;  // query blocks from the tile's first key on
  const int n_steps = p.G * n_q;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  const uint32_t sK = base;
  auto stage = [&](int s) { return base + Cfg::TILE_BYTES + s * Cfg::KV_STAGE; };
  const Bars<STAGES> bars{base + Cfg::TILE_BYTES + STAGES * Cfg::KV_STAGE};
  Tail* tl = reinterpret_cast<Tail*>(smem_raw + (bars.slot() - raw_addr));

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmQk);
    tma_prefetch_desc(&tmDOk);
    tma_prefetch_desc(&tmQm);
    tma_prefetch_desc(&tmDOm);
    bars.init();
    tl->issued = tl->consumed = tl->tile_pending = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    tmem_alloc(bars.slot(), Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tl->tmem;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer: the key tile, then Q / dO blocks in both layouts
      tl->tile_pending = 1;
      mbar_arrive_expect_tx(bars.tile_full(), Cfg::TILE_BYTES);
      tma_load_3d(sK, &tmK, bars.tile_full(), 0, row0 + k0, hk * (HD / 32));
      for (int t = 0; t < n_steps; ++t) {
        const int s = t % STAGES, r = t / STAGES;
        if (r > 0 && !mbar_wait(bars.empty(s), (r - 1) & 1, p.err, kErrWaitEmpty)) break;
        const int h = hk * p.G + t / n_q;
        const int qrow = row0 + k0 + (t % n_q) * BLK;  // rows past the sequence are masked
        const int xb = h * (HD / 32);
        const uint32_t st = stage(s);
        mbar_arrive_expect_tx(bars.full(s), Cfg::KV_STAGE);
        tma_load_3d(st, &tmQk, bars.full(s), 0, qrow, xb);
        tma_load_3d(st + BB, &tmDOk, bars.full(s), 0, qrow, xb);
        tma_load_3d(st + 2 * BB, &tmQm, bars.full(s), 0, qrow, xb);
        tma_load_3d(st + 3 * BB, &tmDOm, bars.full(s), 0, qrow, xb);
        tl->issued = t + 1;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- UMMA issuer
      constexpr uint32_t idesc_s = idesc_tf32(TILE, BLK, false, false);
      constexpr uint32_t idesc_g = idesc_tf32(TILE, HD, false, true);
      bool ok = mbar_wait(bars.tile_full(), 0, p.err, kErrWaitFull);
      if (ok) tl->tile_pending = 0;
      ok = ok && mbar_wait(bars.opnd_ready(), 0, p.err, kErrWaitAccum);
      auto issue_s = [&](int t) -> bool {
        const int s = t % STAGES, bb = t & 1, u = t >> 1;
        if (!mbar_wait(bars.full(s), (t / STAGES) & 1, p.err, kErrWaitFull)) return false;
        tl->consumed = t + 1;
        if (u > 0 && !mbar_wait(bars.s_free(bb), (u - 1) & 1, p.err, kErrWaitAccum)) return false;
        tc_fence_after();
        const uint32_t st = stage(s);
#pragma unroll
        for (int kk = 0; kk < HD / 8; ++kk)  // S^T = K Q^T
          umma_tf32(tmem + s_col(bb), kmajor_desc(sK, TILE, kk), kmajor_desc(st, BLK, kk), idesc_s,
                    kk > 0 ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < HD / 8; ++kk)  // dP^T = V dO^T, V in TMEM
          umma_tf32_ts(tmem + dp_col(bb), tmem + Cfg::OPND_COL + kk * 8, kmajor_desc(st + BB, BLK, kk), idesc_s,
                       kk > 0 ? 1u : 0u);
        umma_commit(bars.s_full(bb));
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int t = 0; ok && t < n_steps; ++t) {
        if (t + 1 < n_steps && !issue_s(t + 1)) break;
        const int s = t % STAGES, bb = t & 1;
        if (!mbar_wait(bars.p_full(bb), (t >> 1) & 1, p.err, kErrWaitAccum)) break;
        tc_fence_after();
        const uint32_t st = stage(s);
#pragma unroll
        for (int kk = 0; kk < BLK / 8; ++kk) {
          const uint32_t acc = (t > 0 || kk > 0) ? 1u : 0u;
          umma_tf32_ts(tmem + Cfg::ACC_COL, tmem + s_col(bb) + kk * 8, mnmajor_desc(st + 3 * BB, kk), idesc_g,
                       acc);  // dV += P dO
          umma_tf32_ts(tmem + Cfg::ACC2_COL, tmem + dp_col(bb) + kk * 8, mnmajor_desc(st + 2 * BB, kk), idesc_g,
                       acc);  // dK += dS Q
        }
        umma_commit(bars.empty(s));
        umma_commit(bars.s_free(bb));
      }
      umma_commit(bars.acc_done());
    }
  } else {
    // ---------------- V into TMEM, softmax gradient, epilogue (lane = key).
    // Steps carry no state from one to the next, so warpgroup grp (warps 2-5,
    // 6-9) takes the steps t = grp mod 2, which use S/dP buffer grp.
    const int grp = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const int key = k0 + row;
    const bool key_ok = key < p.T;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    row_to_tmem<HD>(p.tm_src + static_cast<long long>(row0 + key) * p.ld_in + static_cast<long long>(hk) * HD,
                    key_ok, tmem + lane_base + Cfg::OPND_COL, grp);
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(bars.opnd_ready());
    bool ok = true;
    for (int t = grp; t < n_steps; t += 2) {
      const int bb = grp;
      const int h = hk * p.G + t / n_q;
      const int qs = k0 + (t % n_q) * BLK;
      const long long lrow = (static_cast<long long>(b) * p.H + h) * p.T;
      float l2[32], dl[32];
      load32(p.lse + lrow + qs, p.T - qs, kLog2e, l2);
      load32(p.delta + lrow + qs, p.T - qs, 1.0f, dl);
      if (!mbar_wait(bars.s_full(bb), (t >> 1) & 1, p.err, kErrWaitAccum)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sv[32], dv[32];
      tmem_ld_32x32b_x32(tmem + lane_base + s_col(bb), sv);
      tmem_ld_32x32b_x32(tmem + lane_base + dp_col(bb), dv);
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int q = qs + i;
        const bool keep = q < p.T && key <= q;
        const float pv = keep ? ex2_approx(fmaf(__uint_as_float(sv[i]), p.scale_log2, -l2[i])) : 0.0f;
        sv[i] = __float_as_uint(pv);
        dv[i] = __float_as_uint(pv * (__uint_as_float(dv[i]) - dl[i]) * p.scale);
      }
      tmem_st_32x32b_x32(tmem + lane_base + s_col(bb), sv);
      tmem_st_32x32b_x32(tmem + lane_base + dp_col(bb), dv);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bars.p_full(bb));
    }
    if (ok && mbar_wait(bars.acc_done(), 0, p.err, kErrWaitAccum)) {
      tc_fence_after();
      const long long r = row0 + key;
      if (grp == 0)
        tmem_to_row<HD>(tmem + lane_base + Cfg::ACC_COL, p.out2 + r * p.ld_out2 + static_cast<long long>(hk) * HD,
                        key_ok, 1.0f);
      else
        tmem_to_row<HD>(tmem + lane_base + Cfg::ACC2_COL, p.out + r * p.ld_out + static_cast<long long>(hk) * HD,
                        key_ok, 1.0f);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) drain<STAGES>(bars, tl, p.err);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::TMEM_COLS);
  }
  __syncthreads();
}

// ------------------------------------------------------------------ dQ
template <int HD>
__global__ void __launch_bounds__(BTHREADS, 1)
    flash_bwd_q_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmKk,
                       const __grid_constant__ CUtensorMap tmVk, const __grid_constant__ CUtensorMap tmKm,
                       BwdParams p) {
  using Cfg = BwdCfg<HD>;
  constexpr int STAGES = Cfg::Q_STAGES;
  constexpr int BB = Cfg::BLK_BYTES;
  const int qt = p.n_tiles - 1 - static_cast<int>(blockIdx.x) / p.BHx;  // most keys first
  const int bh = static_cast<int>(blockIdx.x) % p.BHx;
  const int b = bh / p.H, h = bh % p.H, hk = h / p.G;
  const int q0 = qt * TILE;
  const int row0 = b * p.T;
  const int n_kv = (min(p.T, q0 + TILE) + BLK - 1) / BLK;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  const uint32_t sQ = base;
  auto stage = [&](int s) { return base + Cfg::TILE_BYTES + s * Cfg::Q_STAGE; };
  const Bars<STAGES> bars{base + Cfg::TILE_BYTES + STAGES * Cfg::Q_STAGE};
  Tail* tl = reinterpret_cast<Tail*>(smem_raw + (bars.slot() - raw_addr));

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmKk);
    tma_prefetch_desc(&tmVk);
    tma_prefetch_desc(&tmKm);
    bars.init();
    tl->issued = tl->consumed = tl->tile_pending = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    tmem_alloc(bars.slot(), Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tl->tmem;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer: the query tile, then K (both layouts) and V blocks
      tl->tile_pending = 1;
      mbar_arrive_expect_tx(bars.tile_full(), Cfg::TILE_BYTES);
      tma_load_3d(sQ, &tmQ, bars.tile_full(), 0, row0 + q0, h * (HD / 32));
      for (int j = 0; j < n_kv; ++j) {
        const int s = j % STAGES, r = j / STAGES;
        if (r > 0 && !mbar_wait(bars.empty(s), (r - 1) & 1, p.err, kErrWaitEmpty)) break;
        const int krow = row0 + j * BLK;  // keys past the sequence follow every query: masked
        const int xb = hk * (HD / 32);
        const uint32_t st = stage(s);
        mbar_arrive_expect_tx(bars.full(s), Cfg::Q_STAGE);
        tma_load_3d(st, &tmKk, bars.full(s), 0, krow, xb);
        tma_load_3d(st + BB, &tmVk, bars.full(s), 0, krow, xb);
        tma_load_3d(st + 2 * BB, &tmKm, bars.full(s), 0, krow, xb);
        tl->issued = j + 1;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- UMMA issuer
      constexpr uint32_t idesc_s = idesc_tf32(TILE, BLK, false, false);
      constexpr uint32_t idesc_g = idesc_tf32(TILE, HD, false, true);
      bool ok = mbar_wait(bars.tile_full(), 0, p.err, kErrWaitFull);
      if (ok) tl->tile_pending = 0;
      ok = ok && mbar_wait(bars.opnd_ready(), 0, p.err, kErrWaitAccum);
      auto issue_s = [&](int j) -> bool {
        const int s = j % STAGES, bb = j & 1, u = j >> 1;
        if (!mbar_wait(bars.full(s), (j / STAGES) & 1, p.err, kErrWaitFull)) return false;
        tl->consumed = j + 1;
        if (u > 0 && !mbar_wait(bars.s_free(bb), (u - 1) & 1, p.err, kErrWaitAccum)) return false;
        tc_fence_after();
        const uint32_t st = stage(s);
#pragma unroll
        for (int kk = 0; kk < HD / 8; ++kk)  // S = Q K^T
          umma_tf32(tmem + s_col(bb), kmajor_desc(sQ, TILE, kk), kmajor_desc(st, BLK, kk), idesc_s,
                    kk > 0 ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < HD / 8; ++kk)  // dP = dO V^T, dO in TMEM
          umma_tf32_ts(tmem + dp_col(bb), tmem + Cfg::OPND_COL + kk * 8, kmajor_desc(st + BB, BLK, kk), idesc_s,
                       kk > 0 ? 1u : 0u);
        umma_commit(bars.s_full(bb));
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; ok && j < n_kv; ++j) {
        if (j + 1 < n_kv && !issue_s(j + 1)) break;
        const int s = j % STAGES, bb = j & 1;
        if (!mbar_wait(bars.p_full(bb), (j >> 1) & 1, p.err, kErrWaitAccum)) break;
        tc_fence_after();
        const uint32_t st = stage(s);
#pragma unroll
        for (int kk = 0; kk < BLK / 8; ++kk)  // dQ += dS K
          umma_tf32_ts(tmem + Cfg::ACC_COL, tmem + dp_col(bb) + kk * 8, mnmajor_desc(st + 2 * BB, kk), idesc_g,
                       (j > 0 || kk > 0) ? 1u : 0u);
        umma_commit(bars.empty(s));
        umma_commit(bars.s_free(bb));
      }
      umma_commit(bars.acc_done());
    }
  } else {
    // ---------------- dO into TMEM, softmax gradient, epilogue (lane = query);
    // warpgroup grp takes the key blocks j = grp mod 2 (S/dP buffer grp)
    const int grp = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const int q = q0 + row;
    const bool q_ok = q < p.T;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    row_to_tmem<HD>(p.tm_src + static_cast<long long>(row0 + q) * p.ld_in + static_cast<long long>(h) * HD, q_ok,
                    tmem + lane_base + Cfg::OPND_COL, grp);
    const long long li = static_cast<long long>(bh) * p.T + q;
    const float lse2 = q_ok ? p.lse[li] * kLog2e : 0.0f;
    const float dlt = q_ok ? p.delta[li] : 0.0f;
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(bars.opnd_ready());
    bool ok = true;
    for (int j = grp; j < n_kv; j += 2) {
      const int bb = grp;
      if (!mbar_wait(bars.s_full(bb), (j >> 1) & 1, p.err, kErrWaitAccum)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sv[32], dv[32];
      tmem_ld_32x32b_x32(tmem + lane_base + s_col(bb), sv);
      tmem_ld_32x32b_x32(tmem + lane_base + dp_col(bb), dv);
      const int kb = j * BLK;
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const bool keep = q_ok && kb + i <= q;
        const float pv = keep ? ex2_approx(fmaf(__uint_as_float(sv[i]), p.scale_log2, -lse2)) : 0.0f;
        dv[i] = __float_as_uint(pv * (__uint_as_float(dv[i]) - dlt) * p.scale);
      }
      tmem_st_32x32b_x32(tmem + lane_base + dp_col(bb), dv);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bars.p_full(bb));
    }
    if (ok && mbar_wait(bars.acc_done(), 0, p.err, kErrWaitAccum)) {
      tc_fence_after();
      tmem_to_row<HD>(tmem + lane_base + Cfg::ACC_COL,
                      p.out + static_cast<long long>(row0 + q) * p.ld_out + static_cast<long long>(h) * HD, q_ok,
                      1.0f, grp, 2);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) drain<STAGES>(bars, tl, p.err);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::TMEM_COLS);
  }
  __syncthreads();
}

// ------------------------------------------------------------------ CTA pairs
// The same two kernels with a cluster of two CTAs per 256-row tile (keys for
// dK/dV, queries for dQ). The leader issues every UMMA with M = 256
// (cta_group::2); the streamed operand of every product is split between the
// pair (half of its rows for the K-major use, half of the hd columns for the
// MN-major use), so the pair reads each streamed block from L2 once.
constexpr int PBLK_KV = 32;  // queries per step of the dK/dV pair kernel (UMMA N; 16 rows per CTA)
constexpr int PBLK_Q = 64;   // keys per step of the dQ pair kernel (UMMA N; 32 rows per CTA)

template <int HD>
struct PairBwdCfg {
  static constexpr int TILE_BYTES = TILE * HD * 4;
  static constexpr int KV_HALF_K = (PBLK_KV / 2) * HD * 4;  // Q or dO rows, K-major
  static constexpr int KV_HALF_M = PBLK_KV * (HD / 2) * 4;  // Q or dO hd/2 columns, MN-major
  static constexpr int KV_STAGE = 2 * KV_HALF_K + 2 * KV_HALF_M;
  static constexpr int Q_HALF_K = (PBLK_Q / 2) * HD * 4;    // K or V rows, K-major
  static constexpr int Q_HALF_M = PBLK_Q * (HD / 2) * 4;    // K hd/2 columns, MN-major
  static constexpr int Q_STAGE = 2 * Q_HALF_K + Q_HALF_M;
  static constexpr int KV_FIT = (210 * 1024 - TILE_BYTES) / KV_STAGE;
  static constexpr int Q_FIT = (210 * 1024 - TILE_BYTES) / Q_STAGE;
  static constexpr int KV_STAGES = KV_FIT > 4 ? 4 : KV_FIT;
  static constexpr int Q_STAGES = Q_FIT > 4 ? 4 : Q_FIT;
  // after the barriers: a 32 x 16 output staging tile per softmax warp
  static constexpr int STAGE_OUT = 8 * 2048;
  static constexpr int KV_SMEM = TILE_BYTES + KV_STAGES * KV_STAGE + 1024 + 256 + STAGE_OUT;
  static constexpr int Q_SMEM = TILE_BYTES + Q_STAGES * Q_STAGE + 1024 + 256 + STAGE_OUT;
  // TMEM: S (or P) and dP (or dS) buffers, two of each, then the TMEM operand
  // (V or dO) and the accumulators
  static constexpr uint32_t KV_OPND = 4 * PBLK_KV, KV_DV = KV_OPND + HD, KV_DK = KV_DV + HD;
  static constexpr uint32_t Q_OPND = 4 * PBLK_Q, Q_DQ = Q_OPND + HD;
  static constexpr uint32_t TMEM_COLS = 512;
  static_assert(KV_DK + HD <= TMEM_COLS && Q_DQ + HD <= TMEM_COLS, "TMEM budget");
  static_assert(KV_STAGES >= 2 && Q_STAGES >= 2, "two stages");
};

// Barriers of a pair kernel. Those the UMMA issuers wait on are used in the
// leader only; stage-empty, S-full, dP-full and accumulator-done ones receive
// commits multicast to both CTAs.
template <int STAGES>
struct PairBars {
  uint32_t base;
  __device__ uint32_t tile_full() const { return base; }
  __device__ uint32_t full(int s) const { return base + 8u * (1 + s); }
  __device__ uint32_t empty(int s) const { return base + 8u * (1 + STAGES + s); }
  __device__ uint32_t s_full(int bb) const { return base + 8u * (1 + 2 * STAGES + bb); }
  __device__ uint32_t p_full(int bb) const { return base + 8u * (3 + 2 * STAGES + bb); }
  // S (P) part and dP (dS) part of buffer bb no longer read by an UMMA: freed
  // separately, so the next product into one part overlaps the UMMAs still
  // reading the other
  __device__ uint32_t s_free(int bb) const { return base + 8u * (5 + 2 * STAGES + bb); }
  __device__ uint32_t dp_free(int bb) const { return base + 8u * (7 + 2 * STAGES + bb); }
  __device__ uint32_t opnd_ready() const { return base + 8u * (9 + 2 * STAGES); }
  __device__ uint32_t acc_done() const { return base + 8u * (10 + 2 * STAGES); }
  // the dP (dP^T) product of buffer bb complete (S-full covers the S product)
  __device__ uint32_t dp_full(int bb) const { return base + 8u * (11 + 2 * STAGES + bb); }
  __device__ uint32_t slot() const { return base + 8u * (13 + 2 * STAGES); }
  __device__ void init() const {
    mbar_init(tile_full(), 1);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full(s), 1);
      mbar_init(empty(s), 1);
    }
    for (int bb = 0; bb < 2; ++bb) {
      mbar_init(s_full(bb), 1);
      mbar_init(dp_full(bb), 1);
      mbar_init(p_full(bb), 8);  // one warpgroup of each CTA
      mbar_init(s_free(bb), 1);
      mbar_init(dp_free(bb), 1);
    }
    mbar_init(opnd_ready(), 16);  // every softmax warp of both CTAs
    mbar_init(acc_done(), 1);
  }
};

// MN-major descriptor of step kk (8 rows) in a tile of `rows`-row 32-column blocks.
__device__ __forceinline__ uint64_t mnmajor_desc_rows(uint32_t tile, int rows, int kk) {
  return smem_desc(tile + kk * 1024, rows * 128, 512, kLayoutSw128Base32);
}

template <int STAGES>
__device__ __forceinline__ void pair_teardown(bool leader, const PairBars<STAGES>& bars, Tail* tl, int* err,
                                              int warp, uint32_t tmem) {
  tc_fence_before();
  cluster_sync();  // both CTAs are done with their TMEM and with each other's barriers
  if (leader && threadIdx.x == 0) drain<STAGES>(bars, tl, err);
  cluster_sync();  // the pair's copies in flight (after a timeout) have landed
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 512);
  }
}

// ---------------- dK, dV (pair of 128-key tiles)
// Three UMMA issuers in the leader: warp 1 issues each step's S^T, warp 11 its
// dP^T and warp 10 its dV and dK products, so the many small UMMAs of a step are
// issued from three threads (one issuer was the limit).
constexpr int PAIR_BWD_THREADS = BTHREADS + 64;

template <int HD>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(PAIR_BWD_THREADS, 1)
    flash_bwd_kv_pair_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmQk,
                             const __grid_constant__ CUtensorMap tmDOk, const __grid_constant__ CUtensorMap tmQm,
                             const __grid_constant__ CUtensorMap tmDOm, BwdParams p) {
  using Cfg = PairBwdCfg<HD>;
  constexpr int STAGES = Cfg::KV_STAGES;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = static_cast<int>(blockIdx.x) / 2;
  const int kt = pair / p.BHx;  // low key tiles see the most queries: first
  const int bhk = pair % p.BHx;
  const int b = bhk / p.Hkv, hk = bhk % p.Hkv;
  const int k0 = kt * 2 * TILE;
  const int my_k0 = k0 + static_cast<int>(rank) * TILE;
  const int row0 = b * p.T;
  const int n_q = (p.T - k0 + PBLK_KV - 1) / PBLK_KV;
  const int n_steps = p.G * n_q;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  const uint32_t sK = base;
  auto stage = [&](int s) { return base + Cfg::TILE_BYTES + s * Cfg::KV_STAGE; };
  const PairBars<STAGES> bars{base + Cfg::TILE_BYTES + STAGES * Cfg::KV_STAGE};
  Tail* tl = reinterpret_cast<Tail*>(smem_raw + (bars.slot() - raw_addr));

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmQk);
    tma_prefetch_desc(&tmDOk);
    tma_prefetch_desc(&tmQm);
    tma_prefetch_desc(&tmDOm);
    bars.init();
    tl->issued = tl->consumed = tl->tile_pending = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    tmem_alloc_pair(bars.slot(), Cfg::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = tl->tmem;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer (both CTAs): completions land on the leader's barriers
      if (leader) {
        tl->tile_pending = 1;
        mbar_arrive_expect_tx(bars.tile_full(), 2 * Cfg::TILE_BYTES);
      }
      tma_load_3d_pair(sK, &tmK, mapa_shared(bars.tile_full(), 0), 0, row0 + my_k0, hk * (HD / 32));
      for (int t = 0; t < n_steps; ++t) {
        const int s = t % STAGES, r = t / STAGES;
        if (r > 0 && !mbar_wait(bars.empty(s), (r - 1) & 1, p.err, kErrWaitEmpty)) break;
        if (leader) mbar_arrive_expect_tx(bars.full(s), 2 * Cfg::KV_STAGE);
        const int h = hk * p.G + t / n_q;
        const int qrow = row0 + k0 + (t % n_q) * PBLK_KV;  // rows past the sequence are masked
        const int xb = h * (HD / 32);
        const uint32_t st = stage(s);
        const uint32_t fb = mapa_shared(bars.full(s), 0);
        const int half = static_cast<int>(rank) * (PBLK_KV / 2);
        tma_load_3d_pair(st, &tmQk, fb, 0, qrow + half, xb);
        tma_load_3d_pair(st + Cfg::KV_HALF_K, &tmDOk, fb, 0, qrow + half, xb);
        const int xm = xb + static_cast<int>(rank) * (HD / 64);
        tma_load_3d_pair(st + 2 * Cfg::KV_HALF_K, &tmQm, fb, 0, qrow, xm);
        tma_load_3d_pair(st + 2 * Cfg::KV_HALF_K + Cfg::KV_HALF_M, &tmDOm, fb, 0, qrow, xm);
        tl->issued = t + 1;
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ---------------- UMMA issuer A (leader only), M = 256 keys across the pair:
      // S^T of every step
      constexpr uint32_t idesc_s = idesc_tf32(2 * TILE, PBLK_KV, false, false);
      const uint64_t dk0 = kmajor_desc(sK, TILE, 0);
      const bool ok = mbar_wait(bars.tile_full(), 0, p.err, kErrWaitFull);
      if (ok) tl->tile_pending = 0;
      for (int t = 0; ok && t < n_steps; ++t) {
        const int s = t % STAGES, bb = t & 1, u = t >> 1;
        if (!mbar_wait(bars.full(s), (t / STAGES) & 1, p.err, kErrWaitFull)) break;
        tl->consumed = t + 1;
        if (u > 0 && !mbar_wait(bars.s_free(bb), (u - 1) & 1, p.err, kErrWaitAccum)) break;
        tc_fence_after();
        const uint64_t dq0 = kmajor_desc(stage(s), PBLK_KV / 2, 0);
#pragma unroll
        for (int kk = 0; kk < HD / 8; ++kk)  // S^T = K Q^T
          umma_tf32_pair(tmem + s_col_of(bb, PBLK_KV), desc_add(dk0, kchunk_off(TILE, kk)),
                         desc_add(dq0, kchunk_off(PBLK_KV / 2, kk)), idesc_s, kk > 0 ? 1u : 0u);
        umma_commit_pair(bars.s_full(bb), 0x3);
      }
    }
  } else if (warp == 11) {
    if (lane == 0 && leader) {
      // ---------------- UMMA issuer C (leader only): dP^T = V dO^T of every step, V in TMEM
      constexpr uint32_t idesc_s = idesc_tf32(2 * TILE, PBLK_KV, false, false);
      const bool ok = mbar_wait(bars.opnd_ready(), 0, p.err, kErrWaitAccum);
      for (int t = 0; ok && t < n_steps; ++t) {
        const int s = t % STAGES, bb = t & 1, u = t >> 1;
        if (!mbar_wait(bars.full(s), (t / STAGES) & 1, p.err, kErrWaitFull)) break;
        if (u > 0 && !mbar_wait(bars.dp_free(bb), (u - 1) & 1, p.err, kErrWaitAccum)) break;
        tc_fence_after();
        const uint64_t ddo0 = kmajor_desc(stage(s) + Cfg::KV_HALF_K, PBLK_KV / 2, 0);
#pragma unroll
        for (int kk = 0; kk < HD / 8; ++kk)
          umma_tf32_ts_pair(tmem + dp_col_of(bb, PBLK_KV), tmem + Cfg::KV_OPND + kk * 8,
                            desc_add(ddo0, kchunk_off(PBLK_KV / 2, kk)), idesc_s, kk > 0 ? 1u : 0u);
        umma_commit_pair(bars.dp_full(bb), 0x3);
      }
    }
  } else if (warp == 10) {
    if (lane == 0 && leader) {
      // ---------------- UMMA issuer B (leader only): dV += P dO, dK += dS Q of every
      // step once its softmax is done (which implies its S^T and dP^T completed)
      constexpr uint32_t idesc_g = idesc_tf32(2 * TILE, HD, false, true);
      for (int t = 0; t < n_steps; ++t) {
        const int s = t % STAGES, bb = t & 1;
        if (!mbar_wait(bars.p_full(bb), (t >> 1) & 1, p.err, kErrWaitAccum)) break;
        if (!mbar_wait(bars.full(s), (t / STAGES) & 1, p.err, kErrWaitFull)) break;
        tc_fence_after();
        const uint32_t st = stage(s);
        const uint64_t ddom0 = mnmajor_desc_rows(st + 2 * Cfg::KV_HALF_K + Cfg::KV_HALF_M, PBLK_KV, 0);
        const uint64_t dqm0 = mnmajor_desc_rows(st + 2 * Cfg::KV_HALF_K, PBLK_KV, 0);
#pragma unroll
        for (int kk = 0; kk < PBLK_KV / 8; ++kk)  // dV += P dO
          umma_tf32_ts_pair(tmem + Cfg::KV_DV, tmem + s_col_of(bb, PBLK_KV) + kk * 8, desc_add(ddom0, kk * 1024),
                            idesc_g, (t > 0 || kk > 0) ? 1u : 0u);
        umma_commit_pair(bars.s_free(bb), 0x1);
#pragma unroll
        for (int kk = 0; kk < PBLK_KV / 8; ++kk)  // dK += dS Q
          umma_tf32_ts_pair(tmem + Cfg::KV_DK, tmem + dp_col_of(bb, PBLK_KV) + kk * 8, desc_add(dqm0, kk * 1024),
                            idesc_g, (t > 0 || kk > 0) ? 1u : 0u);
        umma_commit_pair(bars.dp_free(bb), 0x1);
        umma_commit_pair(bars.empty(s), 0x3);
      }
      umma_commit_pair(bars.acc_done(), 0x3);
    }
  } else {
    // ---------------- V into TMEM, softmax gradient, epilogue (lane = key);
    // warpgroup grp takes the steps t = grp mod 2 (buffers grp)
    const int grp = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const int key = my_k0 + row;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    float4* wst = reinterpret_cast<float4*>(smem_raw + (bars.base - raw_addr) + 256) + (warp - 2) * 128;
    rows_to_tmem<HD>(p.tm_src + static_cast<long long>(row0) * p.ld_in + static_cast<long long>(hk) * HD, p.ld_in,
                     my_k0 + quarter * 32, p.T, tmem + lane_base + Cfg::KV_OPND, wst, grp);
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive_remote(mapa_shared(bars.opnd_ready(), 0));
    const uint32_t p_full_lead = mapa_shared(bars.p_full(grp), 0);
    bool ok = true;
    for (int t = grp; t < n_steps; t += 2) {
      const int h = hk * p.G + t / n_q;
      const int qs = k0 + (t % n_q) * PBLK_KV;
      const long long lrow = (static_cast<long long>(b) * p.H + h) * p.T;
      float l2[32], dl[32];
      load32(p.lse + lrow + qs, p.T - qs, kLog2e, l2);
      load32(p.delta + lrow + qs, p.T - qs, 1.0f, dl);
      if (!mbar_wait(bars.s_full(grp), (t >> 1) & 1, p.err, kErrWaitAccum) ||
          !mbar_wait(bars.dp_full(grp), (t >> 1) & 1, p.err, kErrWaitAccum)) {
        ok = false;
        break;
      }
      tc_fence_after();
      // S^T and dP^T of this buffer are adjacent: columns [0, 32) and [32, 64)
      uint32_t sd[64];
      tmem_ld_32x32b_x64(tmem + lane_base + s_col_of(grp, PBLK_KV), sd);
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int q = qs + i;
        const bool keep = q < p.T && key <= q;
        const float pv = keep ? ex2_approx(fmaf(__uint_as_float(sd[i]), p.scale_log2, -l2[i])) : 0.0f;
        sd[i] = __float_as_uint(pv);
        sd[32 + i] = __float_as_uint(pv * (__uint_as_float(sd[32 + i]) - dl[i]) * p.scale);
      }
      tmem_st_32x32b_x64(tmem + lane_base + s_col_of(grp, PBLK_KV), sd);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(p_full_lead);
    }
    if (ok && mbar_wait(bars.acc_done(), 0, p.err, kErrWaitAccum)) {
      tc_fence_after();
      if (grp == 0)
        tmem_to_rows<HD>(tmem + lane_base + Cfg::KV_DV,
                         p.out2 + static_cast<long long>(row0) * p.ld_out2 + static_cast<long long>(hk) * HD, p.ld_out2,
                         my_k0 + quarter * 32, p.T, wst);
      else
        tmem_to_rows<HD>(tmem + lane_base + Cfg::KV_DK,
                         p.out + static_cast<long long>(row0) * p.ld_out + static_cast<long long>(hk) * HD, p.ld_out,
                         my_k0 + quarter * 32, p.T, wst);
    }
  }
  pair_teardown<STAGES>(leader, bars, tl, p.err, warp, tmem);
}

// ---------------- dQ (pair of 128-query tiles)
// Three UMMA issuers in the leader as in the dK/dV kernel: warp 1 issues S,
// warp 11 dP and warp 10 the dQ products.
template <int HD>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(PAIR_BWD_THREADS, 1)
    flash_bwd_q_pair_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmKk,
                            const __grid_constant__ CUtensorMap tmVk, const __grid_constant__ CUtensorMap tmKm,
                            BwdParams p) {
  using Cfg = PairBwdCfg<HD>;
  constexpr int STAGES = Cfg::Q_STAGES;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = static_cast<int>(blockIdx.x) / 2;
  const int qt = p.n_tiles - 1 - pair / p.BHx;  // most keys first
  const int bh = pair % p.BHx;
  const int b = bh / p.H, h = bh % p.H, hk = h / p.G;
  const int q0 = qt * 2 * TILE;
  const int my_q0 = q0 + static_cast<int>(rank) * TILE;
  const int row0 = b * p.T;
  const int n_kv = (min(p.T, q0 + 2 * TILE) + PBLK_Q - 1) / PBLK_Q;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  const uint32_t sQ = base;
  auto stage = [&](int s) { return base + Cfg::TILE_BYTES + s * Cfg::Q_STAGE; };
  const PairBars<STAGES> bars{base + Cfg::TILE_BYTES + STAGES * Cfg::Q_STAGE};
  Tail* tl = reinterpret_cast<Tail*>(smem_raw + (bars.slot() - raw_addr));

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmKk);
    tma_prefetch_desc(&tmVk);
    tma_prefetch_desc(&tmKm);
    bars.init();
    tl->issued = tl->consumed = tl->tile_pending = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    tmem_alloc_pair(bars.slot(), Cfg::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = tl->tmem;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer (both CTAs)
      if (leader) {
        tl->tile_pending = 1;
        mbar_arrive_expect_tx(bars.tile_full(), 2 * Cfg::TILE_BYTES);
      }
      tma_load_3d_pair(sQ, &tmQ, mapa_shared(bars.tile_full(), 0), 0, row0 + my_q0, h * (HD / 32));
      for (int j = 0; j < n_kv; ++j) {
        const int s = j % STAGES, r = j / STAGES;
        if (r > 0 && !mbar_wait(bars.empty(s), (r - 1) & 1, p.err, kErrWaitEmpty)) break;
        if (leader) mbar_arrive_expect_tx(bars.full(s), 2 * Cfg::Q_STAGE);
        const int krow = row0 + j * PBLK_Q;  // keys past the sequence follow every query: masked
        const int xb = hk * (HD / 32);
        const uint32_t st = stage(s);
        const uint32_t fb = mapa_shared(bars.full(s), 0);
        const int half = static_cast<int>(rank) * (PBLK_Q / 2);
        tma_load_3d_pair(st, &tmKk, fb, 0, krow + half, xb);
        tma_load_3d_pair(st + Cfg::Q_HALF_K, &tmVk, fb, 0, krow + half, xb);
        tma_load_3d_pair(st + 2 * Cfg::Q_HALF_K, &tmKm, fb, 0, krow, xb + static_cast<int>(rank) * (HD / 64));
        tl->issued = j + 1;
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ---------------- UMMA issuer A (leader only), M = 256 queries across the pair:
      // S of every key block
      constexpr uint32_t idesc_s = idesc_tf32(2 * TILE, PBLK_Q, false, false);
      const uint64_t dqt0 = kmajor_desc(sQ, TILE, 0);
      const bool ok = mbar_wait(bars.tile_full(), 0, p.err, kErrWaitFull);
      if (ok) tl->tile_pending = 0;
      for (int j = 0; ok && j < n_kv; ++j) {
        const int s = j % STAGES, bb = j & 1, u = j >> 1;
        if (!mbar_wait(bars.full(s), (j / STAGES) & 1, p.err, kErrWaitFull)) break;
        tl->consumed = j + 1;
        // the S part was last read by the softmax of block j - 2 (its p_full)
        if (u > 0 && !mbar_wait(bars.p_full(bb), (u - 1) & 1, p.err, kErrWaitAccum)) break;
        tc_fence_after();
        const uint64_t dkk0 = kmajor_desc(stage(s), PBLK_Q / 2, 0);
#pragma unroll
        for (int kk = 0; kk < HD / 8; ++kk)  // S = Q K^T
          umma_tf32_pair(tmem + s_col_of(bb, PBLK_Q), desc_add(dqt0, kchunk_off(TILE, kk)),
                         desc_add(dkk0, kchunk_off(PBLK_Q / 2, kk)), idesc_s, kk > 0 ? 1u : 0u);
        umma_commit_pair(bars.s_full(bb), 0x3);
      }
    }
  } else if (warp == 11) {
    if (lane == 0 && leader) {
      // ---------------- UMMA issuer C (leader only): dP = dO V^T of every key block,
      // dO in TMEM; the dP part was last read by dQ(j - 2) (dp_free)
      constexpr uint32_t idesc_s = idesc_tf32(2 * TILE, PBLK_Q, false, false);
      const bool ok = mbar_wait(bars.opnd_ready(), 0, p.err, kErrWaitAccum);
      for (int j = 0; ok && j < n_kv; ++j) {
        const int s = j % STAGES, bb = j & 1, u = j >> 1;
        if (!mbar_wait(bars.full(s), (j / STAGES) & 1, p.err, kErrWaitFull)) break;
        if (u > 0 && !mbar_wait(bars.dp_free(bb), (u - 1) & 1, p.err, kErrWaitAccum)) break;
        tc_fence_after();
        const uint64_t dvk0 = kmajor_desc(stage(s) + Cfg::Q_HALF_K, PBLK_Q / 2, 0);
#pragma unroll
        for (int kk = 0; kk < HD / 8; ++kk)
          umma_tf32_ts_pair(tmem + dp_col_of(bb, PBLK_Q), tmem + Cfg::Q_OPND + kk * 8,
                            desc_add(dvk0, kchunk_off(PBLK_Q / 2, kk)), idesc_s, kk > 0 ? 1u : 0u);
        umma_commit_pair(bars.dp_full(bb), 0x3);
      }
    }
  } else if (warp == 10) {
    if (lane == 0 && leader) {
      // ---------------- UMMA issuer B (leader only): dQ += dS K of every key block
      // once its softmax is done (which implies its S and dP completed)
      constexpr uint32_t idesc_g = idesc_tf32(2 * TILE, HD, false, true);
      for (int j = 0; j < n_kv; ++j) {
        const int s = j % STAGES, bb = j & 1;
        if (!mbar_wait(bars.p_full(bb), (j >> 1) & 1, p.err, kErrWaitAccum)) break;
        if (!mbar_wait(bars.full(s), (j / STAGES) & 1, p.err, kErrWaitFull)) break;
        tc_fence_after();
        const uint32_t st = stage(s);
        const uint64_t dkm0 = mnmajor_desc_rows(st + 2 * Cfg::Q_HALF_K, PBLK_Q, 0);
#pragma unroll
        for (int kk = 0; kk < PBLK_Q / 8; ++kk)  // dQ += dS K
          umma_tf32_ts_pair(tmem + Cfg::Q_DQ, tmem + dp_col_of(bb, PBLK_Q) + kk * 8, desc_add(dkm0, kk * 1024),
                            idesc_g, (j > 0 || kk > 0) ? 1u : 0u);
        umma_commit_pair(bars.dp_free(bb), 0x1);
        umma_commit_pair(bars.empty(s), 0x3);
      }
      umma_commit_pair(bars.acc_done(), 0x3);
    }
  } else {
    // ---------------- dO into TMEM, softmax gradient, epilogue (lane = query);
    // warpgroup grp takes the key blocks j = grp mod 2
    const int grp = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const int q = my_q0 + row;
    const bool q_ok = q < p.T;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    float4* wst = reinterpret_cast<float4*>(smem_raw + (bars.base - raw_addr) + 256) + (warp - 2) * 128;
    rows_to_tmem<HD>(p.tm_src + static_cast<long long>(row0) * p.ld_in + static_cast<long long>(h) * HD, p.ld_in,
                     my_q0 + quarter * 32, p.T, tmem + lane_base + Cfg::Q_OPND, wst, grp);
    const long long li = static_cast<long long>(bh) * p.T + q;
    const float lse2 = q_ok ? p.lse[li] * kLog2e : 0.0f;
    const float dlt = q_ok ? p.delta[li] : 0.0f;
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive_remote(mapa_shared(bars.opnd_ready(), 0));
    const uint32_t p_full_lead = mapa_shared(bars.p_full(grp), 0);
    bool ok = true;
    for (int j = grp; j < n_kv; j += 2) {
      if (!mbar_wait(bars.s_full(grp), (j >> 1) & 1, p.err, kErrWaitAccum) ||
          !mbar_wait(bars.dp_full(grp), (j >> 1) & 1, p.err, kErrWaitAccum)) {
        ok = false;
        break;
      }
      tc_fence_after();
      {
        // S and dP of this buffer are adjacent: columns [0, 64) and [64, 128)
        uint32_t sd[2 * PBLK_Q];
        tmem_ld_32x32b_x128(tmem + lane_base + s_col_of(grp, PBLK_Q), sd);
        const int kb = j * PBLK_Q;
        uint32_t ds[PBLK_Q];
#pragma unroll
        for (int i = 0; i < PBLK_Q; ++i) {
          const bool keep = q_ok && kb + i <= q;
          const float pv = keep ? ex2_approx(fmaf(__uint_as_float(sd[i]), p.scale_log2, -lse2)) : 0.0f;
          ds[i] = __float_as_uint(pv * (__uint_as_float(sd[PBLK_Q + i]) - dlt) * p.scale);
        }
        tmem_st_32x32b_x64(tmem + lane_base + dp_col_of(grp, PBLK_Q), ds);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(p_full_lead);
    }
    if (ok && mbar_wait(bars.acc_done(), 0, p.err, kErrWaitAccum)) {
      tc_fence_after();
      tmem_to_rows<HD>(tmem + lane_base + Cfg::Q_DQ,
                       p.out + static_cast<long long>(row0) * p.ld_out + static_cast<long long>(h) * HD, p.ld_out,
                       my_q0 + quarter * 32, p.T, wst, grp, 2);
    }
  }
  pair_teardown<STAGES>(leader, bars, tl, p.err, warp, tmem);
}

bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

// Token-major operand [rows, ld]: 3-D view (32 columns, token row, 32-column
// block) whose box brings `box_rows` rows of one head as hd/32 chunks.
void head_map(CUtensorMap* map, const float* ptr, long long rows, long long ld, int heads, int hd, int box_rows,
              bool mn_major, int box_blocks = 0) {
  const long long dims[3] = {32, rows, static_cast<long long>(heads) * hd / 32};
  const long long strides[2] = {ld, 32};
  const int box[3] = {32, box_rows, box_blocks ? box_blocks : hd / 32};
  if (encode_tensor_map(map, ptr, 3, dims, strides, box, mn_major))
    throw std::runtime_error("flash attention backward: tensor map rejected");
}

template <class K>
void set_smem(K kern, int bytes) {
  const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess)
    throw std::runtime_error(std::string("flash attention backward: shared memory size: ") + cudaGetErrorString(e));
}

// At least this much dynamic shared memory, so that one CTA (holding all 512
// TMEM columns) runs per SM and no second CTA waits in tcgen05.alloc.
constexpr int kMinSmem = 120 * 1024;

template <int HD>
void launch_bwd(const AttnShape& s, const float* q, const float* k, const float* v, const float* lse,
                const float* dout, long long lddo, float* dq, float* dk, float* dv, const float* delta, int* d_err,
                cudaStream_t stream) {
  using Cfg = BwdCfg<HD>;
  const long long rows = static_cast<long long>(s.B) * s.T;
  const int n_tiles = (s.T + TILE - 1) / TILE;
  BwdParams p{};
  p.T = s.T;
  p.H = s.H;
  p.Hkv = s.Hkv;
  p.G = s.H / s.Hkv;
  p.n_tiles = n_tiles;
  p.lse = lse;
  p.delta = delta;
  p.scale = s.scale;
  p.scale_log2 = s.scale * kLog2e;
  p.err = d_err;

  {  // dK, dV
    CUtensorMap tk, tqk, tdok, tqm, tdom;
    head_map(&tk, k, rows, s.ldk, s.Hkv, HD, TILE, false);
    head_map(&tqk, q, rows, s.ldq, s.H, HD, BLK, false);
    head_map(&tdok, dout, rows, lddo, s.H, HD, BLK, false);
    head_map(&tqm, q, rows, s.ldq, s.H, HD, BLK, true);
    head_map(&tdom, dout, rows, lddo, s.H, HD, BLK, true);
    BwdParams pk = p;
    pk.BHx = s.B * s.Hkv;
    pk.ld_in = s.ldv;
    pk.tm_src = v;
    pk.out = dk;
    pk.ld_out = s.ldk;
    pk.out2 = dv;
    pk.ld_out2 = s.ldv;
    const int smem = Cfg::KV_SMEM > kMinSmem ? Cfg::KV_SMEM : kMinSmem;
    set_smem(flash_bwd_kv_kernel<HD>, smem);
    const long long grid = static_cast<long long>(n_tiles) * pk.BHx;
    flash_bwd_kv_kernel<HD><<<static_cast<unsigned>(grid), BTHREADS, smem, stream>>>(tk, tqk, tdok, tqm, tdom, pk);
  }
  {  // dQ
    CUtensorMap tq, tkk, tvk, tkm;
    head_map(&tq, q, rows, s.ldq, s.H, HD, TILE, false);
    head_map(&tkk, k, rows, s.ldk, s.Hkv, HD, BLK, false);
    head_map(&tvk, v, rows, s.ldv, s.Hkv, HD, BLK, false);
    head_map(&tkm, k, rows, s.ldk, s.Hkv, HD, BLK, true);
    BwdParams pq = p;
    pq.BHx = s.B * s.H;
    pq.ld_in = lddo;
    pq.tm_src = dout;
    pq.out = dq;
    pq.ld_out = s.ldq;
    const int smem = Cfg::Q_SMEM > kMinSmem ? Cfg::Q_SMEM : kMinSmem;
    set_smem(flash_bwd_q_kernel<HD>, smem);
    const long long grid = static_cast<long long>(n_tiles) * pq.BHx;
    flash_bwd_q_kernel<HD><<<static_cast<unsigned>(grid), BTHREADS, smem, stream>>>(tq, tkk, tvk, tkm, pq);
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess)
    throw std::runtime_error(std::string("flash attention backward launch: ") + cudaGetErrorString(e));
}

template <int HD>
void launch_bwd_pair(const AttnShape& s, const float* q, const float* k, const float* v, const float* lse,
                     const float* dout, long long lddo, float* dq, float* dk, float* dv, const float* delta,
                     int* d_err, cudaStream_t stream, const BwdSide* side) {
  using Cfg = PairBwdCfg<HD>;
  const long long rows = static_cast<long long>(s.B) * s.T;
  const int n_pairs = (s.T + 2 * TILE - 1) / (2 * TILE);
  BwdParams p{};
  p.T = s.T;
  p.H = s.H;
  p.Hkv = s.Hkv;
  p.G = s.H / s.Hkv;
  p.n_tiles = n_pairs;
  p.lse = lse;
  p.delta = delta;
  p.scale = s.scale;
  p.scale_log2 = s.scale * kLog2e;
  p.err = d_err;
  {  // dK, dV
    CUtensorMap tk, tqk, tdok, tqm, tdom;
    head_map(&tk, k, rows, s.ldk, s.Hkv, HD, TILE, false);
    head_map(&tqk, q, rows, s.ldq, s.H, HD, PBLK_KV / 2, false);
    head_map(&tdok, dout, rows, lddo, s.H, HD, PBLK_KV / 2, false);
    head_map(&tqm, q, rows, s.ldq, s.H, HD, PBLK_KV, true, HD / 64);
    head_map(&tdom, dout, rows, lddo, s.H, HD, PBLK_KV, true, HD / 64);
    BwdParams pk = p;
    pk.BHx = s.B * s.Hkv;
    pk.ld_in = s.ldv;
    pk.tm_src = v;
    pk.out = dk;
    pk.ld_out = s.ldk;
    pk.out2 = dv;
    pk.ld_out2 = s.ldv;
    set_smem(flash_bwd_kv_pair_kernel<HD>, Cfg::KV_SMEM);
    const long long grid = 2ll * n_pairs * pk.BHx;
    flash_bwd_kv_pair_kernel<HD>
        <<<static_cast<unsigned>(grid), PAIR_BWD_THREADS, Cfg::KV_SMEM, stream>>>(tk, tqk, tdok, tqm, tdom, pk);
  }
  {  // dQ
    CUtensorMap tq, tkk, tvk, tkm;
    head_map(&tq, q, rows, s.ldq, s.H, HD, TILE, false);
    head_map(&tkk, k, rows, s.ldk, s.Hkv, HD, PBLK_Q / 2, false);
    head_map(&tvk, v, rows, s.ldv, s.Hkv, HD, PBLK_Q / 2, false);
    head_map(&tkm, k, rows, s.ldk, s.Hkv, HD, PBLK_Q, true, HD / 64);
    BwdParams pq = p;
    pq.BHx = s.B * s.H;
    pq.ld_in = lddo;
    pq.tm_src = dout;
    pq.out = dq;
    pq.ld_out = s.ldq;
    set_smem(flash_bwd_q_pair_kernel<HD>, Cfg::Q_SMEM);
    const long long grid = 2ll * n_pairs * pq.BHx;
    // on the side stream the dQ kernel's blocks fill the SMs the dK/dV kernel's
    // last wave leaves idle (the two kernels are independent)
    const cudaStream_t qs = side ? side->stream : stream;
    flash_bwd_q_pair_kernel<HD><<<static_cast<unsigned>(grid), PAIR_BWD_THREADS, Cfg::Q_SMEM, qs>>>(tq, tkk, tvk, tkm,
                                                                                               pq);
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess)
    throw std::runtime_error(std::string("flash attention backward launch: ") + cudaGetErrorString(e));
}

}  // namespace

void attention_backward_flash(const AttnShape& s, const float* q, const float* k, const float* v, const float* o,
                              const float* lse, const float* dout, long long lddo, float* dq, float* dk, float* dv,
                              float* delta, int* d_err, cudaStream_t stream, const BwdSide* side) {
  if (!attention_flash_supported(s) || lddo % 4 != 0 || !aligned16(q) || !aligned16(k) || !aligned16(v) ||
      !aligned16(dout) || !aligned16(dq) || !aligned16(dk) || !aligned16(dv))
    throw std::runtime_error("flash attention backward: unsupported head_dim, stride or alignment");
  attention_delta(s, o, dout, lddo, delta, stream);
  if (side && s.hd != 32) {
    if (cudaEventRecord(side->ready, stream) != cudaSuccess ||
        cudaStreamWaitEvent(side->stream, side->ready, 0) != cudaSuccess)
      throw std::runtime_error("flash attention backward: side stream");
  }
  switch (s.hd) {
    case 32: launch_bwd<32>(s, q, k, v, lse, dout, lddo, dq, dk, dv, delta, d_err, stream); break;
    case 64: launch_bwd_pair<64>(s, q, k, v, lse, dout, lddo, dq, dk, dv, delta, d_err, stream, side); break;
    default: launch_bwd_pair<128>(s, q, k, v, lse, dout, lddo, dq, dk, dv, delta, d_err, stream, side); break;
  }
  if (side && s.hd != 32) {
    if (cudaEventRecord(side->done, side->stream) != cudaSuccess ||
        cudaStreamWaitEvent(stream, side->done, 0) != cudaSuccess)
      throw std::runtime_error("flash attention backward: side stream");
  }
}

}  // namespace mm
