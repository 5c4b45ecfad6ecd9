// TF32 tensor-core GEMM for sm_100a: TMA loads into 128-byte-swizzled shared
// memory, tcgen05.mma (kind::tf32) accumulating in TMEM, tcgen05.ld epilogue.
//
//   C[m, n] = sum_k A(m, k) * B(n, k)   (+ R[m, n] when R is given)
//
// Each operand is either K-major (A(m, k) = A[m * lda + k], the contraction index
// contiguous) or MN-major (A(m, k) = A[k * lda + m]). The three products of a
// linear layer map onto this as follows (X [tokens x in], W [in x out], row-major
// as crates/midman-tensor/src/ops_matmul.rs:55-75 stores them):
//   Y  = X W      : A = X  K-major,  B = W  MN-major
//   dX = dY W^T   : A = dY K-major,  B = W  K-major   (kernels.rs:66-75 gemm_nt)
//   dW = X^T dY   : A = X  MN-major, B = dY MN-major  (kernels.rs:78-84 gemm_tn)
//
// The batched form (grid.z = batch) addresses every operand through a 4-D tensor
// map (inner, head, row, batch), so per-head slices of token-major activations
// and grouped-query key/value heads are read in place; it also restricts the
// work to the causal part of an attention product (tiles above the diagonal
// skipped, or the K loop cut at the diagonal).
//
// Warp roles (192 threads; a persistent grid of at most one CTA per SM, each
// walking BM x BN output tiles with a stride of the grid size):
//   warp 0      TMA producer (one lane), STAGES-deep ring of A/B stages
//   warp 1      TMEM allocator + UMMA issuer (one lane), two TMEM accumulators
//   warps 2..5  epilogue: TMEM -> registers -> global (optionally + R), which
//               overlaps the UMMAs of the CTA's next tile
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdint>
#include <cstdio>
#include <mutex>

#include "gemm.h"
#include "ptx.cuh"
#include "tma.h"

namespace mm {

namespace {

constexpr int BM = 128;
constexpr int BK = 32;  // 32 fp32 = 128 bytes = one swizzle row
constexpr int A_STAGE_BYTES = BM * BK * 4;  // 16 KB
constexpr int THREADS = 192;
constexpr int SMEM_BUDGET = 196608;  // operand ring; leaves room for barriers and alignment

template <int BN>
struct Tile {
  static constexpr int B_STAGE_BYTES = BN * BK * 4;
  static constexpr int STAGE_BYTES = A_STAGE_BYTES + B_STAGE_BYTES;
  static constexpr int STAGES = SMEM_BUDGET / STAGE_BYTES > 8 ? 8 : SMEM_BUDGET / STAGE_BYTES;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers, slot, counters*/ +
                                    4 * 32 * 32 * 4 /*epilogue staging, one 32x32 tile per epilogue warp*/;
};

// Byte offset of the 4 KB block that holds MN columns [32j, 32j+32) of an
// MN-major tile; its 32 K-rows sit 128 bytes apart.
constexpr uint32_t MN_BLOCK_BYTES = BK * 128;

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int32_t x,
                                            int32_t h, int32_t y, int32_t b) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(h), "r"(y), "r"(b)
      : "memory");
}

template <bool BATCHED>
__device__ __forceinline__ void load_box(uint32_t dst, const CUtensorMap* map, uint32_t bar, int32_t x, int32_t y,
                                         int32_t zh, int32_t zb) {
  if (BATCHED)
    tma_load_4d(dst, map, bar, x, zh, y, zb);
  else
    tma_load_2d(dst, map, bar, x, y);
}

// Output tile t of this launch: batch, m block, n block (m fastest, so CTAs that
// run at the same time share B tiles and walk down A), and its K range.
struct TileInfo {
  int z, m0, n0, kt_begin, n_k;
  bool skip;
};

template <int BN, bool BATCHED>
__device__ __forceinline__ TileInfo tile_info(int t, int M, int N, int K, const GemmBatch& bt) {
  const int tm = (M + BM - 1) / BM, tn = (N + BN - 1) / BN;
  TileInfo ti;
  ti.z = t / (tm * tn);
  const int r = t % (tm * tn);
  ti.m0 = (r % tm) * BM;
  ti.n0 = (r / tm) * BN;
  ti.skip = BATCHED && bt.causal == kCausalSkipUpper && ti.n0 > ti.m0 + BM - 1;  // above the diagonal
  int kt_begin = 0, k_end = K;
  if (BATCHED && bt.causal == kCausalKBelow) k_end = min(K, ti.m0 + BM - bt.k_off);
  if (BATCHED && bt.causal == kCausalKAbove) kt_begin = max(0, ti.m0 - bt.k_off) / BK;
  const int kt_end = (k_end + BK - 1) / BK;
  ti.kt_begin = kt_begin;
  ti.n_k = kt_end > kt_begin ? kt_end - kt_begin : 0;
  if (BATCHED && bt.skip_empty && ti.n_k == 0) ti.skip = true;  // C += 0: nothing to write
  return ti;
}

// Epilogue of one warp for its 32 rows (starting at wrow0) of a BM x BN tile:
// the accumulator slice at TMEM address `acc` (lane = row) goes through the
// warp's staging tile to C (+ R). As soon as the last TMEM slice is loaded the
// warp arrives on `release_bar` (in the pair's leader CTA when `remote`), which
// frees the accumulator for the tile after next.
__device__ __forceinline__ void release(uint32_t bar, bool remote) {
  if (remote)
    mbar_arrive_remote(bar);
  else
    mbar_arrive(bar);
}

template <int BN>
__device__ __forceinline__ void store_tile(uint32_t acc, bool has_k, float4* stage_tile, int wrow0, int n0, float* Ct,
                                           long long ldc, const float* R, long long ldr, int M, int N,
                                           uint32_t release_bar, bool remote) {
  const int lane = threadIdx.x % 32;
  bool released = false;
  if (has_k) {
    // Each 32-column slice goes TMEM -> registers (lane = row) -> this warp's
    // staging tile -> global with 8 lanes per row, so every R load and C
    // store instruction covers four whole 128-byte row segments. The
    // residual of slice c + 1 is loaded before slice c is stored (slices
    // are disjoint, so this holds when R aliases C).
    const int sub = lane & 7, rsub = lane >> 3;
    float4 rnext[8];
    auto load_r = [&](int c) {
      const int col = n0 + c * 32 + 4 * sub;
#pragma unroll
      for (int it = 0; it < 8; ++it) {
        const int row = wrow0 + it * 4 + rsub;
        rnext[it] = (col + 3 < N && row < M)
                        ? *reinterpret_cast<const float4*>(R + static_cast<long long>(row) * ldr + col)
                        : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    };
    if (R) load_r(0);
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      uint32_t r[32];
      tmem_ld_32x32b_x32(acc + c * 32, r);
      if (c == BN / 32 - 1) {  // the accumulator is free for the tile after next
        tc_fence_before();
        __syncwarp();
        if (lane == 0) release(release_bar, remote);
        released = true;
      }
      // 4-float granules, XOR-swizzled by row: conflict-free both ways
#pragma unroll
      for (int g = 0; g < 8; ++g)
        stage_tile[lane * 8 + (g ^ (lane & 7))] =
            make_float4(__uint_as_float(r[4 * g]), __uint_as_float(r[4 * g + 1]), __uint_as_float(r[4 * g + 2]),
                        __uint_as_float(r[4 * g + 3]));
      __syncwarp();
      float4 v[8];
#pragma unroll
      for (int it = 0; it < 8; ++it) {
        const int rr = it * 4 + rsub;
        v[it] = stage_tile[rr * 8 + (sub ^ (rr & 7))];
        if (R) {
          v[it].x += rnext[it].x; v[it].y += rnext[it].y; v[it].z += rnext[it].z; v[it].w += rnext[it].w;
        }
      }
      if (R && c + 1 < BN / 32) load_r(c + 1);
      const int col = n0 + c * 32 + 4 * sub;
#pragma unroll
      for (int it = 0; it < 8; ++it) {
        const int row = wrow0 + it * 4 + rsub;
        if (row >= M || col >= N) continue;
        float* cp = Ct + static_cast<long long>(row) * ldc + col;
        if (col + 3 < N) {
          *reinterpret_cast<float4*>(cp) = v[it];
        } else {  // ragged right edge: the residual was not prefetched
          const float* rp = R ? R + static_cast<long long>(row) * ldr + col : nullptr;
          const float vv[4] = {v[it].x, v[it].y, v[it].z, v[it].w};
          for (int e = 0; e < 4 && col + e < N; ++e) cp[e] = vv[e] + (rp ? rp[e] : 0.0f);
        }
      }
      __syncwarp();  // before the next slice overwrites the staging tile
    }
  } else {
    // Empty K range: the product is zero, C = R (or 0).
    const int row = wrow0 + lane;
    if (row < M)
      for (int col = n0; col < n0 + BN && col < N; ++col)
        Ct[static_cast<long long>(row) * ldc + col] = R ? R[static_cast<long long>(row) * ldr + col] : 0.0f;
  }
  if (!released) {
    tc_fence_before();
    __syncwarp();
    if (lane == 0) release(release_bar, remote);
  }
}

// Persistent: each CTA walks tiles blockIdx.x, blockIdx.x + gridDim.x, ... The
// TMA/UMMA stage ring runs across tile boundaries, and the accumulator is
// double-buffered in TMEM, so the epilogue of one tile overlaps the MMAs of the
// next.
template <bool A_MN, bool B_MN, int BN, bool BATCHED>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_tf32_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, float* C,
                     long long ldc, const float* R, long long ldr, int M, int N, int K, int* err, GemmBatch bt,
                     int total_tiles, int mn3d) {
  using TL = Tile<BN>;
  constexpr int STAGES = TL::STAGES;
  constexpr int STAGE_BYTES = TL::STAGE_BYTES;
  constexpr uint32_t ACC_COLS = 2 * BN;  // two accumulators

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;  // SW128 atoms want 1024-byte alignment
  uint8_t* smem = smem_raw + (base - raw_addr);

  const uint32_t bar_base = base + STAGES * STAGE_BYTES;
  auto full_bar = [&](int s) { return bar_base + 8u * s; };
  auto empty_bar = [&](int s) { return bar_base + 8u * (STAGES + s); };
  auto acc_full = [&](int b) { return bar_base + 8u * (2 * STAGES + b); };
  auto acc_empty = [&](int b) { return bar_base + 8u * (2 * STAGES + 2 + b); };
  const uint32_t tmem_slot = bar_base + 8u * (2 * STAGES + 4);
  uint8_t* tail = smem + STAGES * STAGE_BYTES + 8 * (2 * STAGES + 4);
  uint32_t* tmem_slot_ptr = reinterpret_cast<uint32_t*>(tail);
  // Stages loaded by the producer and consumed by the UMMA issuer; they differ
  // only when a wait timed out, and teardown then drains the difference.
  int* loads_issued = reinterpret_cast<int*>(tail + 8);
  int* loads_consumed = loads_issued + 1;

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    if (K > 0) {  // with K = 0 the maps are not built (the tiles are R or zeros)
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
    }
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(acc_full(b), 1);
      mbar_init(acc_empty(b), 4);  // one arrival per epilogue warp
    }
    *loads_issued = 0;
    *loads_consumed = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, ACC_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot_ptr;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer
      int it = 0;  // stage-ring position, across tiles
      bool ok = true;
      for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
        const TileInfo ti = tile_info<BN, BATCHED>(t, M, N, K, bt);
        if (ti.skip) continue;
        const int a_zb = BATCHED ? ti.z / bt.a_zdiv : 0, a_zh = BATCHED ? (ti.z % bt.a_zdiv) / bt.a_zgroup : 0;
        const int b_zb = BATCHED ? ti.z / bt.b_zdiv : 0, b_zh = BATCHED ? (ti.z % bt.b_zdiv) / bt.b_zgroup : 0;
        for (int i = 0; i < ti.n_k; ++i, ++it) {
          const int s = it % STAGES;
          const int round = it / STAGES;
          if (round > 0 && !mbar_wait(empty_bar(s), (round - 1) & 1, err, kErrWaitEmpty)) {
            ok = false;
            break;
          }
          const uint32_t sa = base + s * STAGE_BYTES;
          const uint32_t sb = sa + A_STAGE_BYTES;
          mbar_arrive_expect_tx(full_bar(s), STAGE_BYTES);
          const int k0 = (ti.kt_begin + i) * BK;
          if (!A_MN) {
            load_box<BATCHED>(sa, &tmA, full_bar(s), k0, ti.m0, a_zh, a_zb);
          } else if (!BATCHED && (mn3d & 1)) {
            tma_load_3d(sa, &tmA, full_bar(s), 0, k0, ti.m0 / 32);
          } else {
#pragma unroll
            for (int j = 0; j < BM / 32; ++j)
              load_box<BATCHED>(sa + j * MN_BLOCK_BYTES, &tmA, full_bar(s), ti.m0 + 32 * j, k0, a_zh, a_zb);
          }
          if (!B_MN) {
            load_box<BATCHED>(sb, &tmB, full_bar(s), k0, ti.n0, b_zh, b_zb);
          } else if (!BATCHED && (mn3d & 2)) {
            tma_load_3d(sb, &tmB, full_bar(s), 0, k0, ti.n0 / 32);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 32; ++j)
              load_box<BATCHED>(sb + j * MN_BLOCK_BYTES, &tmB, full_bar(s), ti.n0 + 32 * j, k0, b_zh, b_zb);
          }
          *loads_issued = it + 1;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- UMMA issuer
      constexpr uint32_t idesc = idesc_tf32(BM, BN, A_MN, B_MN);
      int it = 0, j = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
        const TileInfo ti = tile_info<BN, BATCHED>(t, M, N, K, bt);
        if (ti.skip) continue;
        const int buf = j & 1;
        // the epilogue must have drained this accumulator (tile j - 2)
        if (j >= 2 && !mbar_wait(acc_empty(buf), ((j >> 1) - 1) & 1, err, kErrWaitAccum)) break;
        tc_fence_after();
        const uint32_t acc = tmem_base + buf * BN;
        for (int i = 0; i < ti.n_k; ++i, ++it) {
          const int s = it % STAGES;
          const int round = it / STAGES;
          if (!mbar_wait(full_bar(s), round & 1, err, kErrWaitFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          *loads_consumed = it + 1;
          const uint32_t sa = base + s * STAGE_BYTES;
          const uint32_t sb = sa + A_STAGE_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 8; ++k) {
            // K-major: step 8 tf32 = 32 bytes along the swizzled row.
            // MN-major (32-byte swizzle atoms of 4 K-rows): step 8 K-rows = 1024
            // bytes; LBO = next 32-wide MN block, SBO = next group of 4 K-rows.
            const uint64_t adesc = A_MN ? smem_desc(sa + k * 1024, MN_BLOCK_BYTES, 512, kLayoutSw128Base32)
                                        : smem_desc(sa + k * 32, 16, 1024, kLayoutSw128);
            const uint64_t bdesc = B_MN ? smem_desc(sb + k * 1024, MN_BLOCK_BYTES, 512, kLayoutSw128Base32)
                                        : smem_desc(sb + k * 32, 16, 1024, kLayoutSw128);
            umma_tf32(acc, adesc, bdesc, idesc, (i | k) != 0 ? 1u : 0u);
          }
          umma_commit(empty_bar(s));
        }
        umma_commit(acc_full(buf));  // also when the K range is empty: the epilogue writes R or 0
        ++j;
      }
    }
  } else {
    // ---------------- epilogue: warps 2..5 cover TMEM lane quarters (warp % 4)
    const int quarter = warp & 3;
    float4* stage_tile = reinterpret_cast<float4*>(smem + STAGES * STAGE_BYTES + 256) + quarter * 256;
    int j = 0;
    for (int t = blockIdx.x; t < total_tiles; t += gridDim.x) {
      const TileInfo ti = tile_info<BN, BATCHED>(t, M, N, K, bt);
      if (ti.skip) continue;
      const int buf = j & 1;
      if (!mbar_wait(acc_full(buf), (j >> 1) & 1, err, kErrWaitAccum)) break;
      tc_fence_after();
      float* Ct = C;
      const float* Rt = R;
      if (BATCHED) {
        const long long zoff = (ti.z / bt.c_zdiv) * bt.c_sb + ((ti.z % bt.c_zdiv) / bt.c_zgroup) * bt.c_sh;
        Ct += zoff;
        if (R) Rt += zoff;  // R has C's layout
      }
      store_tile<BN>(tmem_base + buf * BN + (static_cast<uint32_t>(quarter * 32) << 16), ti.n_k > 0, stage_tile,
                     ti.m0 + quarter * 32, ti.n0, Ct, ldc, Rt, ldr, M, N, acc_empty(buf), false);
      ++j;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) {
    // Only after a timed-out wait can a TMA stage still be in flight here: let
    // each one land (bounded) before the CTA's shared memory is released.
    for (int i = *loads_consumed; i < *loads_issued; ++i)
      if (!mbar_wait(full_bar(i % STAGES), (i / STAGES) & 1, err, kErrWaitDrain, 1000000000ull)) break;
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, ACC_COLS);
  }
  __syncthreads();
}

// ------------------------------------------------------------------ CTA pairs
// A cluster of two CTAs computes 256 x 256 output tiles: CTA r loads rows
// m0 + 128 r of A and rows n0 + 128 r of B (its half of the UMMA's N), the
// leader issues M = 256 cta_group::2 UMMAs, and each CTA's TMEM holds the
// accumulator of its 128 rows. Per stage a CTA loads 32 KB (16 KB of A, 16 KB
// of B) for the same MMA work per SM that costs a single CTA 48 KB (A plus a
// 256-wide B), so the ring is deeper (6 stages) and L2 serves a third less.
// Pair tile 256 x PN. Only PN = 256 is launched: 256 x 128 tiles were measured at
// ~400 TF/s against ~650 (each UMMA reads the same A for half the work).
template <int PN>
struct PairTile {
  static constexpr int B_BYTES = (PN / 2) * BK * 4;  // 16 KB (PN 256) or 8 KB
  static constexpr int STAGE = A_STAGE_BYTES + B_BYTES;
  static constexpr int STAGES = PN == 256 ? 6 : 8;
  static constexpr int SMEM = STAGES * STAGE + 1024 + 256 + 4 * 32 * 32 * 4;
  static constexpr int TILE_FLOATS = 2 * BM * PN;
};

constexpr int P_TILE_FLOATS_MAX = 2 * BM * 256;  // one 256 x 256 tile

// Work unit u of a pair launch. Tiles [0, full) are whole units; each of the
// remaining tiles (the last, partial wave) is cut into `splits` parts of its K
// loop, so that the last wave keeps more pairs busy for a shorter time. A part
// writes its partial sum to workspace tile `slot`; split_reduce_kernel adds the
// parts (in order) and the residual into C.
// Pair tile t -> (M tile, N tile). Tiles go in groups of kGroupM M tiles; inside a
// group the M tile changes fastest, then the N tile. The pairs working at the
// same time (74 on 148 SMs) then cover a block of about kGroupM x 9 tiles, so
// they read that block's rows of A and columns of B from L2 while their K steps
// advance together, instead of every row of A once per wave (with the M tile
// fastest over the whole of M, a wave of an M = 8192 product reads all of A:
// measured DRAM traffic 2.0-2.9x the operands' bytes).
constexpr int kGroupM = 8;
__device__ __forceinline__ void pair_tile_mn(int t, int tm, int tn, int& mt, int& nt) {
  const int per_group = kGroupM * tn;
  const int g = t / per_group, r = t - g * per_group;
  const int rows = min(kGroupM, tm - g * kGroupM);
  mt = g * kGroupM + r % rows;
  nt = r / rows;
}

struct PairUnit {
  int tile, kb, ke, slot;  // slot < 0: a whole tile, written to C
};

__device__ __forceinline__ PairUnit pair_unit(int u, int full, int splits, int n_k) {
  PairUnit w;
  if (u < full) {
    w.tile = u;
    w.kb = 0;
    w.ke = n_k;
    w.slot = -1;
  } else {
    const int v = u - full, part = v % splits;
    w.tile = full + v / splits;
    w.kb = (n_k * part) / splits;
    w.ke = (n_k * (part + 1)) / splits;
    w.slot = v;
  }
  return w;
}

// The operands of a pair launch: up to kMaxSegments (A, B) pairs whose products
// are summed into one accumulator (C = sum_s A_s B_s^T), their K steps one after
// another. Each segment has its own tensor maps (a segment's ragged last K step
// reads zeros past its own K) and MN-major box flags (bit 0: A, bit 1: B).
constexpr int kMaxSegments = 3;
struct PairOperands {
  CUtensorMap a[kMaxSegments];
  CUtensorMap b[kMaxSegments];
  int seg_end[kMaxSegments];  // K steps of segments 0..s together
  int mn3d[kMaxSegments];
  int nseg;
};

// Work units reach a pair's roles through a ring of kUnitRing slots in both CTAs'
// shared memory: the leader's producer takes each next unit and publishes it
// (unit_full, one arrival; the peer CTA's slot by a remote store and a
// cluster-scope release arrival), and every other role of the pair (the peer's
// producer, the UMMA issuer, the eight epilogue warps) reads it and frees the
// slot (the leader's unit_empty). -1 ends every role's loop. A pair's first
// unit is its position in the grid; the next ones come from the launch's
// ticket counter (`sched`: tickets, finished pairs) when one is given, so that
// pairs whose SMs were busy when the launch started (another stream's kernel,
// NCCL) take fewer units; otherwise the pair strides by the grid.
constexpr int kUnitRing = 4;
constexpr int kUnitConsumers = 1 + 1 + 8;  // peer producer, UMMA issuer, epilogue warps of both CTAs

template <bool A_MN, bool B_MN, int PN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(THREADS, 1)
    gemm_pair_kernel(const __grid_constant__ PairOperands ops, float* C, long long ldc, const float* R, long long ldr,
                     int M, int N, int* err, int total_tiles, int full_tiles, int splits, float* ws,
                     unsigned int* sched) {
  using Cfg = PairTile<PN>;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = static_cast<int>(blockIdx.x) / 2, npairs = static_cast<int>(gridDim.x) / 2;
  const int tm = (M + 2 * BM - 1) / (2 * BM), tn = (N + PN - 1) / PN;
  const int n_k = ops.seg_end[ops.nseg - 1];
  // The segments' bounds, tensor maps and box flags in registers, read once:
  // segment g covers K steps [seg_end[g-1], seg_end[g]); bounds past nseg are
  // n_k, so steps never select a segment that does not exist.
  static_assert(kMaxSegments == 3, "the selects below assume three segments");
  const int seg_end0 = ops.nseg > 1 ? ops.seg_end[0] : n_k;
  const int seg_end1 = ops.nseg > 2 ? ops.seg_end[1] : n_k;
  const CUtensorMap* map_a0 = &ops.a[0];
  const CUtensorMap* map_a1 = &ops.a[1];
  const CUtensorMap* map_a2 = &ops.a[2];
  const CUtensorMap* map_b0 = &ops.b[0];
  const CUtensorMap* map_b1 = &ops.b[1];
  const CUtensorMap* map_b2 = &ops.b[2];
  const int mn3d0 = ops.mn3d[0], mn3d1 = ops.mn3d[1], mn3d2 = ops.mn3d[2];
  const bool single = ops.nseg == 1;
  const int total_units = full_tiles + (total_tiles - full_tiles) * splits;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw_addr);
  const uint32_t bar_base = base + Cfg::STAGES * Cfg::STAGE;
  auto full_bar = [&](int s) { return bar_base + 8u * s; };
  auto empty_bar = [&](int s) { return bar_base + 8u * (Cfg::STAGES + s); };
  auto acc_full = [&](int b) { return bar_base + 8u * (2 * Cfg::STAGES + b); };
  auto acc_empty = [&](int b) { return bar_base + 8u * (2 * Cfg::STAGES + 2 + b); };
  auto unit_full = [&](int s) { return bar_base + 8u * (2 * Cfg::STAGES + 4 + s); };
  auto unit_empty = [&](int s) { return bar_base + 8u * (2 * Cfg::STAGES + 4 + kUnitRing + s); };
  constexpr int kBars = 2 * Cfg::STAGES + 4 + 2 * kUnitRing;
  const uint32_t tmem_slot = bar_base + 8u * kBars;
  uint8_t* tail = smem + Cfg::STAGES * Cfg::STAGE + 8 * kBars;
  uint32_t* tmem_slot_ptr = reinterpret_cast<uint32_t*>(tail);
  int* loads_issued = reinterpret_cast<int*>(tail + 8);
  int* loads_consumed = loads_issued + 1;
  volatile int* unit_ring = reinterpret_cast<volatile int*>(tail + 16);
  static_assert(8 * kBars + 16 + 4 * kUnitRing <= 256, "barriers and counters fit their 256 bytes");

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    for (int g = 0; g < ops.nseg; ++g) {
      tma_prefetch_desc(&ops.a[g]);
      tma_prefetch_desc(&ops.b[g]);
    }
    for (int s = 0; s < Cfg::STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(acc_full(b), 1);
      mbar_init(acc_empty(b), 8);  // four epilogue warps in each CTA
    }
    for (int s = 0; s < kUnitRing; ++s) {
      mbar_init(unit_full(s), 1);
      mbar_init(unit_empty(s), kUnitConsumers);
    }
    *loads_issued = 0;
    *loads_consumed = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, 2 * PN);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot_ptr;

  // Tickets: the leader takes the ticket of its next unit one unit ahead (the
  // atomic's latency hides behind the current unit's loads). A ticket past the
  // last unit ends the pair and counts it as finished; the last pair to finish
  // resets the counter for the next launch on the stream.
  auto take_ticket = [&]() -> unsigned { return atomicAdd(&sched[0], 1u); };
  auto unit_of_ticket = [&](unsigned ticket) -> int {
    const int v = npairs + static_cast<int>(ticket);
    if (v < total_units) return v;
    __threadfence();
    if (atomicAdd(&sched[1], 1u) == static_cast<unsigned>(npairs - 1)) {
      __threadfence();
      atomicExch(&sched[0], 0u);
      atomicExch(&sched[1], 0u);
    }
    return -1;
  };

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer (both CTAs); completions land on the leader's barriers
      int it = 0, ring_i = 0;
      bool ok = true;
      int u = leader ? pair : -1;
      unsigned ticket = (leader && sched) ? take_ticket() : 0u;  // the unit after u
      for (;;) {
        const int rs = ring_i % kUnitRing, rr = ring_i / kUnitRing;
        if (leader) {  // publish this unit (or the end) to the pair
          if (rr > 0 && !mbar_wait_cluster(unit_empty(rs), (rr - 1) & 1, err, kErrWaitUnit)) {
            ok = false;
            break;
          }
          unit_ring[rs] = u;
          st_shared_cluster(mapa_shared(smem_u32(const_cast<int*>(&unit_ring[rs])), 1), u);
          mbar_arrive(unit_full(rs));
          mbar_arrive_remote_release(mapa_shared(unit_full(rs), 1));
        } else {
          if (!mbar_wait_cluster(unit_full(rs), rr & 1, err, kErrWaitUnit)) {
            ok = false;
            break;
          }
          u = unit_ring[rs];
          mbar_arrive_remote_release(mapa_shared(unit_empty(rs), 0));
        }
        ++ring_i;
        if (u >= total_units) {  // never handed out; guards the workspace index
          atomicCAS(err, 0, kErrWaitUnit);
          u = -1;
        }
        if (u < 0) break;
        const PairUnit w = pair_unit(u, full_tiles, splits, n_k);
        const int t = w.tile;
        int mt, nt;
        pair_tile_mn(t, tm, tn, mt, nt);
        const int my_m0 = mt * 2 * BM + static_cast<int>(rank) * BM;
        const int my_n0 = nt * PN + static_cast<int>(rank) * (PN / 2);
        for (int i = w.kb; i < w.ke; ++i, ++it) {
          const int s = it % Cfg::STAGES, round = it / Cfg::STAGES;
          if (round > 0 && !mbar_wait(empty_bar(s), (round - 1) & 1, err, kErrWaitEmpty)) {
            ok = false;
            break;
          }
          if (leader) mbar_arrive_expect_tx(full_bar(s), 2 * Cfg::STAGE);
          const uint32_t fb = mapa_shared(full_bar(s), 0);
          const uint32_t sa = base + s * Cfg::STAGE, sb = sa + A_STAGE_BYTES;
          // One (A, B) pair: the tensor maps are addressed in the kernel's parameter
          // space directly. Several: the segment of K step i from registers.
          auto issue = [&](const CUtensorMap* tmA, const CUtensorMap* tmB, int mn3d, int k0) {
            if (!A_MN) {
              tma_load_2d_pair(sa, tmA, fb, k0, my_m0);
            } else if (mn3d & 1) {
              tma_load_3d_pair(sa, tmA, fb, 0, k0, my_m0 / 32);
            } else {
#pragma unroll
              for (int j = 0; j < BM / 32; ++j) tma_load_2d_pair(sa + j * MN_BLOCK_BYTES, tmA, fb, my_m0 + 32 * j, k0);
            }
            if (!B_MN) {
              tma_load_2d_pair(sb, tmB, fb, k0, my_n0);
            } else if (mn3d & 2) {
              tma_load_3d_pair(sb, tmB, fb, 0, k0, my_n0 / 32);
            } else {
#pragma unroll
              for (int j = 0; j < PN / 64; ++j)
                tma_load_2d_pair(sb + j * MN_BLOCK_BYTES, tmB, fb, my_n0 + 32 * j, k0);
            }
          };
          if (single) {
            issue(&ops.a[0], &ops.b[0], mn3d0, i * BK);
          } else {
            const int g = (i >= seg_end0 ? 1 : 0) + (i >= seg_end1 ? 1 : 0);
            issue(g == 0 ? map_a0 : g == 1 ? map_a1 : map_a2, g == 0 ? map_b0 : g == 1 ? map_b1 : map_b2,
                  g == 0 ? mn3d0 : g == 1 ? mn3d1 : mn3d2, (i - (g == 0 ? 0 : g == 1 ? seg_end0 : seg_end1)) * BK);
          }
          *loads_issued = it + 1;
        }
        if (!ok) break;
        if (leader) {
          if (!sched) {
            u = u + npairs < total_units ? u + npairs : -1;
          } else {
            u = unit_of_ticket(ticket);
            if (u >= 0) ticket = take_ticket();
          }
        }
      }
      // keep the ticket protocol whole after a timed-out wait: take tickets
      // until this pair's last one
      if (leader && sched && u >= 0) {
        while ((u = unit_of_ticket(ticket)) >= 0) ticket = take_ticket();
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ---------------- UMMA issuer (leader only), M = 256 across the pair
      constexpr uint32_t idesc = idesc_tf32(2 * BM, PN, A_MN, B_MN);
      int it = 0, j = 0, ring_i = 0;
      bool ok = true;
      for (;;) {
        const int rs = ring_i % kUnitRing, rr = ring_i / kUnitRing;
        if (!mbar_wait(unit_full(rs), rr & 1, err, kErrWaitUnit)) break;
        const int u = unit_ring[rs];
        mbar_arrive(unit_empty(rs));
        ++ring_i;
        if (u < 0 || u >= total_units) break;
        const PairUnit w = pair_unit(u, full_tiles, splits, n_k);
        const int buf = j & 1;
        if (j >= 2 && !mbar_wait(acc_empty(buf), ((j >> 1) - 1) & 1, err, kErrWaitAccum)) break;
        tc_fence_after();
        const uint32_t acc = tmem_base + buf * PN;
        for (int i = w.kb; i < w.ke; ++i, ++it) {
          const int s = it % Cfg::STAGES, round = it / Cfg::STAGES;
          if (!mbar_wait(full_bar(s), round & 1, err, kErrWaitFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          *loads_consumed = it + 1;
          const uint32_t sa = base + s * Cfg::STAGE, sb = sa + A_STAGE_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 8; ++k) {
            const uint64_t adesc = A_MN ? smem_desc(sa + k * 1024, MN_BLOCK_BYTES, 512, kLayoutSw128Base32)
                                        : smem_desc(sa + k * 32, 16, 1024, kLayoutSw128);
            const uint64_t bdesc = B_MN ? smem_desc(sb + k * 1024, MN_BLOCK_BYTES, 512, kLayoutSw128Base32)
                                        : smem_desc(sb + k * 32, 16, 1024, kLayoutSw128);
            umma_tf32_pair(acc, adesc, bdesc, idesc, (i != w.kb || k != 0) ? 1u : 0u);
          }
          umma_commit_pair(empty_bar(s), 0x3);
        }
        if (!ok) break;
        umma_commit_pair(acc_full(buf), 0x3);
        ++j;
      }
    }
  } else {
    // ---------------- epilogue (both CTAs): this CTA's 128 rows, all 256 columns
    const int quarter = warp & 3;
    float4* stage_tile = reinterpret_cast<float4*>(smem + Cfg::STAGES * Cfg::STAGE + 256) + quarter * 256;
    int j = 0, ring_i = 0;
    for (;;) {
      const int rs = ring_i % kUnitRing, rr = ring_i / kUnitRing;
      int u = -1;
      if (lane == 0) {
        const bool got = leader ? mbar_wait(unit_full(rs), rr & 1, err, kErrWaitUnit)
                                : mbar_wait_cluster(unit_full(rs), rr & 1, err, kErrWaitUnit);
        if (got) {
          u = unit_ring[rs];
          if (leader)
            mbar_arrive(unit_empty(rs));
          else
            mbar_arrive_remote_release(mapa_shared(unit_empty(rs), 0));
        }
      }
      u = __shfl_sync(0xffffffffu, u, 0);
      ++ring_i;
      if (u < 0 || u >= total_units) break;
      const PairUnit w = pair_unit(u, full_tiles, splits, n_k);
      const int t = w.tile;
      const int buf = j & 1;
      if (!mbar_wait(acc_full(buf), (j >> 1) & 1, err, kErrWaitAccum)) break;
      tc_fence_after();
      const uint32_t acc = tmem_base + buf * PN + (static_cast<uint32_t>(quarter * 32) << 16);
      if (w.slot < 0) {
        int mt, nt;
        pair_tile_mn(t, tm, tn, mt, nt);
        const int my_m0 = mt * 2 * BM + static_cast<int>(rank) * BM;
        store_tile<PN>(acc, true, stage_tile, my_m0 + quarter * 32, nt * PN, C, ldc, R, ldr, M, N,
                        mapa_shared(acc_empty(buf), 0), true);
      } else {  // a K part: the whole 256 x 256 partial tile into its workspace slot
        store_tile<PN>(acc, true, stage_tile, static_cast<int>(rank) * BM + quarter * 32, 0,
                        ws + static_cast<long long>(w.slot) * Cfg::TILE_FLOATS, PN, nullptr, 0, 2 * BM, PN,
                        mapa_shared(acc_empty(buf), 0), true);
      }
      ++j;
    }
  }

  tc_fence_before();
  cluster_sync();  // both CTAs are done with their TMEM and with each other's barriers
  if (leader && threadIdx.x == 0) {
    // after a timed-out wait, let the pair's copies in flight land (bounded)
    for (int i = *loads_consumed; i < *loads_issued; ++i)
      if (!mbar_wait(full_bar(i % Cfg::STAGES), (i / Cfg::STAGES) & 1, err, kErrWaitDrain, 1000000000ull)) break;
  }
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, 2 * PN);
  }
}

// C = sum of a split tile's K parts (in part order) + R. Grid (split tiles,
// 256 / rows per block): a block covers 256 / (PN / 4) rows of one tile, a thread
// 4 columns.
template <int PN>
__global__ void __launch_bounds__(256) split_reduce_kernel(const float* __restrict__ ws, int splits, int full_tiles,
                                                           int tm, float* C, long long ldc, const float* R,
                                                           long long ldr, int M, int N) {
  constexpr int P_TILE_FLOATS = PairTile<PN>::TILE_FLOATS;
  constexpr int ROWS = 256 / (PN / 4);  // rows per block
  const int tl = blockIdx.x, t = full_tiles + tl;
  const int row = blockIdx.y * ROWS + threadIdx.x / (PN / 4), col = (threadIdx.x % (PN / 4)) * 4;
  int mt, nt;
  pair_tile_mn(t, tm, (N + PN - 1) / PN, mt, nt);
  const int gm = mt * 2 * BM + row, gn = nt * PN + col;
  if (gm >= M || gn >= N) return;
  const float* src = ws + static_cast<long long>(tl) * splits * P_TILE_FLOATS + row * PN + col;
  float4 v = *reinterpret_cast<const float4*>(src);
  for (int p = 1; p < splits; ++p) {
    const float4 q = *reinterpret_cast<const float4*>(src + static_cast<long long>(p) * P_TILE_FLOATS);
    v.x += q.x;
    v.y += q.y;
    v.z += q.z;
    v.w += q.w;
  }
  const float vals[4] = {v.x, v.y, v.z, v.w};
  float* cp = C + static_cast<long long>(gm) * ldc + gn;
  const float* rp = R ? R + static_cast<long long>(gm) * ldr + gn : nullptr;
  if (gn + 3 < N) {
    float4 o = v;
    if (rp) {
      const float4 r = *reinterpret_cast<const float4*>(rp);
      o.x += r.x;
      o.y += r.y;
      o.z += r.z;
      o.w += r.w;
    }
    *reinterpret_cast<float4*>(cp) = o;
  } else {
    for (int e = 0; e < 4 && gn + e < N; ++e) cp[e] = vals[e] + (rp ? rp[e] : 0.0f);
  }
}

// ------------------------------------------------------------------ 3xTF32 on CTA pairs
// The exact mode's product, C = sum_k A(m, k) B(n, k) with A = Ah + Al and
// B = Bh + Bl (the hi/lo TF32 copies split_tf32 makes): 256 x 256 tiles on CTA
// pairs as in gemm_pair_kernel, but each stage holds this CTA's 128 rows of all
// four of Ah, Al, Bh, Bl for one K step of 32, and the leader issues Al Bh,
// Ah Bl, Ah Bh (the small terms first) for it. The tensor core's f32
// accumulation loses a little, in the same direction, on every UMMA, so its
// error grows with the number of UMMAs summed into one accumulator: every
// X3_CHUNK K steps (24 UMMAs) start a fresh TMEM accumulator, and the epilogue
// warps add each one into a running sum held in registers (f32, round to
// nearest). The two accumulators alternate, so a chunk's add overlaps the next
// chunk's UMMAs. Eight epilogue warps: warp w reads TMEM lanes 32 (w % 4).. and
// accumulator columns 128 ((w - 2) / 4).., a running sum of 128 floats per
// thread. Units (whole tiles, then the last wave's K parts) and the workspace of
// the parts are those of the TF32 pair kernel; units go to pairs by a fixed
// stride (the exact mode runs on one stream). Registers: each of the SM's four
// 16K-register quarters holds up to three of the ten warps, which caps a
// thread at 168 registers; the sum (128) leaves room for 16-column TMEM loads.
constexpr int X3_THREADS = 320;
constexpr int X3_STAGES = 3;
constexpr int X3_TILE = BM * BK * 4;  // 16 KB: this CTA's rows of one of Ah, Al, Bh, Bl
constexpr int X3_STAGE = 4 * X3_TILE;
constexpr int X3_CHUNK = 2;  // K steps per TMEM accumulation
constexpr int X3_SMEM = X3_STAGES * X3_STAGE + 1024 + 256 + 8 * 32 * 32 * 4;
static_assert(X3_SMEM <= 232448, "3xTF32 pair kernel shared memory");

struct X3Operands {
  CUtensorMap ah[kMaxSegments], al[kMaxSegments], bh[kMaxSegments], bl[kMaxSegments];
  int seg_end[kMaxSegments];  // K steps of segments 0..s together
  int mn3d[kMaxSegments];
  int nseg;
};

// A warp's running sum (its 32 rows, lane = row, and NC columns from n0)
// through the warp's staging tile to C (+ R): 8 lanes per 32-column row
// segment, so every R load and C store instruction covers whole 128-byte
// segments (the layout of store_tile).
template <int NC>
__device__ __forceinline__ void store_sum(const float (&sum)[NC], float4* stage_tile, int wrow0, int n0, float* Ct,
                                          long long ldc, const float* R, long long ldr, int M, int N) {
  static_assert(NC % 32 == 0, "whole 32-column slices");
  const int lane = threadIdx.x % 32, sub = lane & 7, rsub = lane >> 3;
#pragma unroll
  for (int c = 0; c < NC / 32; ++c) {
#pragma unroll
    for (int g = 0; g < 8; ++g)
      stage_tile[lane * 8 + (g ^ (lane & 7))] =
          make_float4(sum[c * 32 + 4 * g], sum[c * 32 + 4 * g + 1], sum[c * 32 + 4 * g + 2], sum[c * 32 + 4 * g + 3]);
    __syncwarp();
    const int col = n0 + c * 32 + 4 * sub;
#pragma unroll 4
    for (int it = 0; it < 8; ++it) {
      const int rr = it * 4 + rsub, row = wrow0 + rr;
      float4 v = stage_tile[rr * 8 + (sub ^ (rr & 7))];
      if (row < M && col < N) {
        float* cp = Ct + static_cast<long long>(row) * ldc + col;
        const float* rp = R ? R + static_cast<long long>(row) * ldr + col : nullptr;
        if (col + 3 < N) {
          if (rp) {
            const float4 r = *reinterpret_cast<const float4*>(rp);
            v.x += r.x;
            v.y += r.y;
            v.z += r.z;
            v.w += r.w;
          }
          *reinterpret_cast<float4*>(cp) = v;
        } else {
          const float vv[4] = {v.x, v.y, v.z, v.w};
          for (int e = 0; e < 4 && col + e < N; ++e) cp[e] = vv[e] + (rp ? rp[e] : 0.0f);
        }
      }
    }
    __syncwarp();  // before the next slice overwrites the staging tile
  }
}

template <bool A_MN, bool B_MN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(X3_THREADS, 1)
    gemm3x_pair_kernel(const __grid_constant__ X3Operands ops, float* C, long long ldc, const float* R, long long ldr,
                       int M, int N, int* err, int total_tiles, int full_tiles, int splits, float* ws) {
  constexpr int PN = 256;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = static_cast<int>(blockIdx.x) / 2, npairs = static_cast<int>(gridDim.x) / 2;
  const int tm = (M + 2 * BM - 1) / (2 * BM), tn = (N + PN - 1) / PN;
  const int n_k = ops.seg_end[ops.nseg - 1];
  const int total_units = full_tiles + (total_tiles - full_tiles) * splits;
  static_assert(kMaxSegments == 3, "the selects below assume three segments");
  const int seg_end0 = ops.nseg > 1 ? ops.seg_end[0] : n_k;
  const int seg_end1 = ops.nseg > 2 ? ops.seg_end[1] : n_k;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw_addr);
  const uint32_t bar_base = base + X3_STAGES * X3_STAGE;
  auto full_bar = [&](int s) { return bar_base + 8u * s; };
  auto empty_bar = [&](int s) { return bar_base + 8u * (X3_STAGES + s); };
  auto acc_full = [&](int b) { return bar_base + 8u * (2 * X3_STAGES + b); };
  auto acc_empty = [&](int b) { return bar_base + 8u * (2 * X3_STAGES + 2 + b); };
  constexpr int kBars = 2 * X3_STAGES + 4;
  const uint32_t tmem_slot = bar_base + 8u * kBars;
  uint8_t* tail = smem + X3_STAGES * X3_STAGE + 8 * kBars;
  uint32_t* tmem_slot_ptr = reinterpret_cast<uint32_t*>(tail);
  int* loads_issued = reinterpret_cast<int*>(tail + 8);
  int* loads_consumed = loads_issued + 1;
  static_assert(8 * kBars + 16 <= 256, "barriers and counters fit their 256 bytes");

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    for (int g = 0; g < ops.nseg; ++g) {
      tma_prefetch_desc(&ops.ah[g]);
      tma_prefetch_desc(&ops.al[g]);
      tma_prefetch_desc(&ops.bh[g]);
      tma_prefetch_desc(&ops.bl[g]);
    }
    for (int s = 0; s < X3_STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(acc_full(b), 1);
      mbar_init(acc_empty(b), 16);  // eight epilogue warps in each CTA
    }
    *loads_issued = 0;
    *loads_consumed = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, 2 * PN);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot_ptr;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer (both CTAs); completions land on the leader's barriers
      int it = 0;
      bool ok = true;
      for (int u = pair; u < total_units && ok; u += npairs) {
        const PairUnit w = pair_unit(u, full_tiles, splits, n_k);
        int mt, nt;
        pair_tile_mn(w.tile, tm, tn, mt, nt);
        const int my_m0 = mt * 2 * BM + static_cast<int>(rank) * BM;
        const int my_n0 = nt * PN + static_cast<int>(rank) * (PN / 2);
        for (int i = w.kb; i < w.ke; ++i, ++it) {
          const int s = it % X3_STAGES, round = it / X3_STAGES;
          if (round > 0 && !mbar_wait(empty_bar(s), (round - 1) & 1, err, kErrWaitEmpty)) {
            ok = false;
            break;
          }
          if (leader) mbar_arrive_expect_tx(full_bar(s), 2 * X3_STAGE);
          const uint32_t fb = mapa_shared(full_bar(s), 0);
          const uint32_t sa = base + s * X3_STAGE;
          const int g = (i >= seg_end0 ? 1 : 0) + (i >= seg_end1 ? 1 : 0);
          const int k0 = (i - (g == 0 ? 0 : g == 1 ? seg_end0 : seg_end1)) * BK;
          const int mn3d = g == 0 ? ops.mn3d[0] : g == 1 ? ops.mn3d[1] : ops.mn3d[2];
          // this CTA's 128 rows (M or N) of one operand copy at K step k0
          auto load = [&](uint32_t dst, const CUtensorMap* map, bool mn, bool box3d, int mn0) {
            if (!mn) {
              tma_load_2d_pair(dst, map, fb, k0, mn0);
            } else if (box3d) {
              tma_load_3d_pair(dst, map, fb, 0, k0, mn0 / 32);
            } else {
#pragma unroll
              for (int j = 0; j < BM / 32; ++j) tma_load_2d_pair(dst + j * MN_BLOCK_BYTES, map, fb, mn0 + 32 * j, k0);
            }
          };
          load(sa, &ops.ah[g], A_MN, mn3d & 1, my_m0);
          load(sa + X3_TILE, &ops.al[g], A_MN, mn3d & 1, my_m0);
          load(sa + 2 * X3_TILE, &ops.bh[g], B_MN, mn3d & 2, my_n0);
          load(sa + 3 * X3_TILE, &ops.bl[g], B_MN, mn3d & 2, my_n0);
          *loads_issued = it + 1;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ---------------- UMMA issuer (leader only), M = 256 across the pair
      constexpr uint32_t idesc = idesc_tf32(2 * BM, PN, A_MN, B_MN);
      int it = 0, j = 0;
      bool ok = true;
      for (int u = pair; u < total_units && ok; u += npairs) {
        const PairUnit w = pair_unit(u, full_tiles, splits, n_k);
        for (int cb = w.kb; cb < w.ke && ok; cb += X3_CHUNK) {
          const int ce = min(w.ke, cb + X3_CHUNK);
          const int buf = j & 1;
          if (j >= 2 && !mbar_wait(acc_empty(buf), ((j >> 1) - 1) & 1, err, kErrWaitAccum)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t acc = tmem_base + buf * PN;
          for (int i = cb; i < ce; ++i, ++it) {
            const int s = it % X3_STAGES, round = it / X3_STAGES;
            if (!mbar_wait(full_bar(s), round & 1, err, kErrWaitFull)) {
              ok = false;
              break;
            }
            tc_fence_after();
            *loads_consumed = it + 1;
            const uint32_t sa = base + s * X3_STAGE;
            // the (A, B) copies of the three terms, small ones first: Al Bh, Ah Bl, Ah Bh
#pragma unroll
            for (int term = 0; term < 3; ++term) {
#pragma unroll
              for (int k = 0; k < BK / 8; ++k) {
                const uint32_t at = sa + (term == 0 ? X3_TILE : 0);
                const uint32_t bt = sa + (term == 1 ? 3 * X3_TILE : 2 * X3_TILE);
                const uint64_t adesc = A_MN ? smem_desc(at + k * 1024, MN_BLOCK_BYTES, 512, kLayoutSw128Base32)
                                            : smem_desc(at + k * 32, 16, 1024, kLayoutSw128);
                const uint64_t bdesc = B_MN ? smem_desc(bt + k * 1024, MN_BLOCK_BYTES, 512, kLayoutSw128Base32)
                                            : smem_desc(bt + k * 32, 16, 1024, kLayoutSw128);
                umma_tf32_pair(acc, adesc, bdesc, idesc, (i != cb || term != 0 || k != 0) ? 1u : 0u);
              }
            }
            umma_commit_pair(empty_bar(s), 0x3);
          }
          if (!ok) break;
          umma_commit_pair(acc_full(buf), 0x3);
          ++j;
        }
      }
    }
  } else {
    // ---------------- epilogue (both CTAs): 32 rows x 128 columns of the tile per warp
    const int quarter = warp & 3, half = (warp - 2) >> 2;
    float4* stage_tile = reinterpret_cast<float4*>(smem + X3_STAGES * X3_STAGE + 256) + (warp - 2) * 256;
    const int srow = static_cast<int>(rank) * BM + quarter * 32;  // this warp's rows of the tile
    int j = 0;
    bool ok = true;
    for (int u = pair; u < total_units && ok; u += npairs) {
      const PairUnit w = pair_unit(u, full_tiles, splits, n_k);
      float sum[128];
#pragma unroll
      for (int e = 0; e < 128; ++e) sum[e] = 0.0f;
      for (int cb = w.kb; cb < w.ke; cb += X3_CHUNK) {
        const int buf = j & 1;
        if (!mbar_wait(acc_full(buf), (j >> 1) & 1, err, kErrWaitAccum)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t acc = tmem_base + buf * PN + (static_cast<uint32_t>(quarter * 32) << 16) + half * 128;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          uint32_t r[16];
          tmem_ld_32x32b_x16(acc + c * 16, r);
#pragma unroll
          for (int e = 0; e < 16; ++e) sum[c * 16 + e] += __uint_as_float(r[e]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(mapa_shared(acc_empty(buf), 0));
        ++j;
      }
      if (!ok) break;
      if (w.slot < 0) {
        int mt, nt;
        pair_tile_mn(w.tile, tm, tn, mt, nt);
        store_sum(sum, stage_tile, mt * 2 * BM + srow, nt * PN + half * 128, C, ldc, R, ldr, M, N);
      } else {  // a K part: its partial sums into the part's workspace tile
        store_sum(sum, stage_tile, srow, half * 128, ws + static_cast<long long>(w.slot) * PairTile<PN>::TILE_FLOATS,
                  PN, nullptr, 0, 2 * BM, PN);
      }
    }
  }

  tc_fence_before();
  cluster_sync();  // both CTAs are done with their TMEM and with each other's barriers
  if (leader && threadIdx.x == 0) {
    // after a timed-out wait, let the pair's copies in flight land (bounded)
    for (int i = *loads_consumed; i < *loads_issued; ++i)
      if (!mbar_wait(full_bar(i % X3_STAGES), (i / X3_STAGES) & 1, err, kErrWaitDrain, 1000000000ull)) break;
  }
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, 2 * PN);
  }
}

// The batched form of the 3xTF32 product (attention's exact mode): one CTA per
// 128 x BN output tile of the batched GEMM (4-D operand views, causal tile
// modes as in gemm_tf32_kernel), each stage holding Ah, Al, Bh, Bl for one K
// step, the three terms issued by one thread, and the same per-chunk
// accumulations summed in the epilogue warps' registers (warp w: TMEM lanes
// 32 (w % 4).., columns (BN / 2) ((w - 2) / 4)..).
template <int BN>
struct X3BatchTile {
  static constexpr int A_BYTES = BM * BK * 4;  // 16 KB
  static constexpr int B_BYTES = BN * BK * 4;
  static constexpr int STAGE = 2 * A_BYTES + 2 * B_BYTES;
  static constexpr int STAGES = 196608 / STAGE > 4 ? 4 : 196608 / STAGE;
  static constexpr int SMEM = STAGES * STAGE + 1024 + 256 + 8 * 32 * 32 * 4;
};

struct X3BatchMaps {
  CUtensorMap ah, al, bh, bl;
};

template <bool A_MN, bool B_MN, int BN>
__global__ void __launch_bounds__(X3_THREADS, 1)
    gemm3x_batched_kernel(const __grid_constant__ X3BatchMaps maps, float* C, long long ldc, const float* R,
                          long long ldr, int M, int N, int K, int* err, GemmBatch bt, int total_tiles) {
  using TL = X3BatchTile<BN>;
  constexpr int STAGES = TL::STAGES;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw_addr);
  const uint32_t bar_base = base + STAGES * TL::STAGE;
  auto full_bar = [&](int s) { return bar_base + 8u * s; };
  auto empty_bar = [&](int s) { return bar_base + 8u * (STAGES + s); };
  auto acc_full = [&](int b) { return bar_base + 8u * (2 * STAGES + b); };
  auto acc_empty = [&](int b) { return bar_base + 8u * (2 * STAGES + 2 + b); };
  constexpr int kBars = 2 * STAGES + 4;
  const uint32_t tmem_slot = bar_base + 8u * kBars;
  uint8_t* tail = smem + STAGES * TL::STAGE + 8 * kBars;
  uint32_t* tmem_slot_ptr = reinterpret_cast<uint32_t*>(tail);
  int* loads_issued = reinterpret_cast<int*>(tail + 8);
  int* loads_consumed = loads_issued + 1;
  static_assert(8 * kBars + 16 <= 256, "barriers and counters fit their 256 bytes");

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&maps.ah);
    tma_prefetch_desc(&maps.al);
    tma_prefetch_desc(&maps.bh);
    tma_prefetch_desc(&maps.bl);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(acc_full(b), 1);
      mbar_init(acc_empty(b), 8);  // one arrival per epilogue warp
    }
    *loads_issued = 0;
    *loads_consumed = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 2 * BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot_ptr;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
        const TileInfo ti = tile_info<BN, true>(t, M, N, K, bt);
        if (ti.skip) continue;
        const int a_zb = ti.z / bt.a_zdiv, a_zh = (ti.z % bt.a_zdiv) / bt.a_zgroup;
        const int b_zb = ti.z / bt.b_zdiv, b_zh = (ti.z % bt.b_zdiv) / bt.b_zgroup;
        for (int i = 0; i < ti.n_k; ++i, ++it) {
          const int s = it % STAGES, round = it / STAGES;
          if (round > 0 && !mbar_wait(empty_bar(s), (round - 1) & 1, err, kErrWaitEmpty)) {
            ok = false;
            break;
          }
          const uint32_t sa = base + s * TL::STAGE, sb = sa + 2 * TL::A_BYTES;
          mbar_arrive_expect_tx(full_bar(s), TL::STAGE);
          const int k0 = (ti.kt_begin + i) * BK;
          auto load_a = [&](uint32_t dst, const CUtensorMap* map) {
            if (!A_MN) {
              load_box<true>(dst, map, full_bar(s), k0, ti.m0, a_zh, a_zb);
            } else {
#pragma unroll
              for (int j = 0; j < BM / 32; ++j)
                load_box<true>(dst + j * MN_BLOCK_BYTES, map, full_bar(s), ti.m0 + 32 * j, k0, a_zh, a_zb);
            }
          };
          auto load_b = [&](uint32_t dst, const CUtensorMap* map) {
            if (!B_MN) {
              load_box<true>(dst, map, full_bar(s), k0, ti.n0, b_zh, b_zb);
            } else {
#pragma unroll
              for (int j = 0; j < BN / 32; ++j)
                load_box<true>(dst + j * MN_BLOCK_BYTES, map, full_bar(s), ti.n0 + 32 * j, k0, b_zh, b_zb);
            }
          };
          load_a(sa, &maps.ah);
          load_a(sa + TL::A_BYTES, &maps.al);
          load_b(sb, &maps.bh);
          load_b(sb + TL::B_BYTES, &maps.bl);
          *loads_issued = it + 1;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- UMMA issuer
      constexpr uint32_t idesc = idesc_tf32(BM, BN, A_MN, B_MN);
      int it = 0, j = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
        const TileInfo ti = tile_info<BN, true>(t, M, N, K, bt);
        if (ti.skip) continue;
        for (int cb = 0; cb < ti.n_k && ok; cb += X3_CHUNK) {
          const int ce = min(ti.n_k, cb + X3_CHUNK);
          const int buf = j & 1;
          if (j >= 2 && !mbar_wait(acc_empty(buf), ((j >> 1) - 1) & 1, err, kErrWaitAccum)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t acc = tmem_base + buf * BN;
          for (int i = cb; i < ce; ++i, ++it) {
            const int s = it % STAGES, round = it / STAGES;
            if (!mbar_wait(full_bar(s), round & 1, err, kErrWaitFull)) {
              ok = false;
              break;
            }
            tc_fence_after();
            *loads_consumed = it + 1;
            const uint32_t sa = base + s * TL::STAGE, sb = sa + 2 * TL::A_BYTES;
            // the (A, B) copies of the three terms, small ones first: Al Bh, Ah Bl, Ah Bh
#pragma unroll
            for (int term = 0; term < 3; ++term) {
#pragma unroll
              for (int k = 0; k < BK / 8; ++k) {
                const uint32_t at = sa + (term == 0 ? TL::A_BYTES : 0);
                const uint32_t bt_ = sb + (term == 1 ? TL::B_BYTES : 0);
                const uint64_t adesc = A_MN ? smem_desc(at + k * 1024, MN_BLOCK_BYTES, 512, kLayoutSw128Base32)
                                            : smem_desc(at + k * 32, 16, 1024, kLayoutSw128);
                const uint64_t bdesc = B_MN ? smem_desc(bt_ + k * 1024, MN_BLOCK_BYTES, 512, kLayoutSw128Base32)
                                            : smem_desc(bt_ + k * 32, 16, 1024, kLayoutSw128);
                umma_tf32(acc, adesc, bdesc, idesc, (i != cb || term != 0 || k != 0) ? 1u : 0u);
              }
            }
            umma_commit(empty_bar(s));
          }
          if (!ok) break;
          umma_commit(acc_full(buf));
          ++j;
        }
      }
    }
  } else {
    // ---------------- epilogue: 32 rows x BN / 2 columns of the tile per warp
    constexpr int NC = BN / 2;
    const int quarter = warp & 3, half = (warp - 2) >> 2;
    float4* stage_tile = reinterpret_cast<float4*>(smem + STAGES * TL::STAGE + 256) + (warp - 2) * 256;
    int j = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
      const TileInfo ti = tile_info<BN, true>(t, M, N, K, bt);
      if (ti.skip) continue;
      float sum[NC];
#pragma unroll
      for (int e = 0; e < NC; ++e) sum[e] = 0.0f;
      for (int cb = 0; cb < ti.n_k; cb += X3_CHUNK) {
        const int buf = j & 1;
        if (!mbar_wait(acc_full(buf), (j >> 1) & 1, err, kErrWaitAccum)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t acc = tmem_base + buf * BN + (static_cast<uint32_t>(quarter * 32) << 16) + half * NC;
#pragma unroll
        for (int c = 0; c < NC / 16; ++c) {
          uint32_t r[16];
          tmem_ld_32x32b_x16(acc + c * 16, r);
#pragma unroll
          for (int e = 0; e < 16; ++e) sum[c * 16 + e] += __uint_as_float(r[e]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(acc_empty(buf));
        ++j;
      }
      if (!ok) break;
      const long long zoff = (ti.z / bt.c_zdiv) * bt.c_sb + ((ti.z % bt.c_zdiv) / bt.c_zgroup) * bt.c_sh;
      store_sum<NC>(sum, stage_tile, ti.m0 + quarter * 32, ti.n0 + half * NC, C + zoff, ldc, R ? R + zoff : nullptr,
                    ldr, M, N);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = *loads_consumed; i < *loads_issued; ++i)
      if (!mbar_wait(full_bar(i % STAGES), (i / STAGES) & 1, err, kErrWaitDrain, 1000000000ull)) break;
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 2 * BN);
  }
  __syncthreads();
}

__device__ __forceinline__ float rn_tf32_dev(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// Writes a warp's 32 rows (lane = row) x NC values through its staging tile as
// TF32 pairs, hi = rn(v) to H and lo = rn(v - hi) to L (8 lanes per 32-column
// row segment, as store_sum).
template <int NC>
__device__ __forceinline__ void store_pair(const float (&val)[NC], float4* stage_tile, int wrow0, int n0, float* H,
                                           float* L, long long ld, int M, int N) {
  const int lane = threadIdx.x % 32, sub = lane & 7, rsub = lane >> 3;
#pragma unroll
  for (int c = 0; c < NC / 32; ++c) {
#pragma unroll
    for (int g = 0; g < 8; ++g)
      stage_tile[lane * 8 + (g ^ (lane & 7))] =
          make_float4(val[c * 32 + 4 * g], val[c * 32 + 4 * g + 1], val[c * 32 + 4 * g + 2], val[c * 32 + 4 * g + 3]);
    __syncwarp();
    const int col = n0 + c * 32 + 4 * sub;
#pragma unroll 2
    for (int it = 0; it < 8; ++it) {
      const int rr = it * 4 + rsub, row = wrow0 + rr;
      const float4 v = stage_tile[rr * 8 + (sub ^ (rr & 7))];
      if (row >= M || col >= N) continue;
      const float4 h = make_float4(rn_tf32_dev(v.x), rn_tf32_dev(v.y), rn_tf32_dev(v.z), rn_tf32_dev(v.w));
      const float4 l = make_float4(rn_tf32_dev(v.x - h.x), rn_tf32_dev(v.y - h.y), rn_tf32_dev(v.z - h.z),
                                   rn_tf32_dev(v.w - h.w));
      const long long off = static_cast<long long>(row) * ld + col;
      if (col + 3 < N) {
        *reinterpret_cast<float4*>(H + off) = h;
        *reinterpret_cast<float4*>(L + off) = l;
      } else {
        const float hh[4] = {h.x, h.y, h.z, h.w}, ll[4] = {l.x, l.y, l.z, l.w};
        for (int e = 0; e < 4 && col + e < N; ++e) {
          H[off + e] = hh[e];
          L[off + e] = ll[e];
        }
      }
    }
    __syncwarp();
  }
}

// The exact-mode attention backward's score tiles in one launch. For every
// causal 128 x BN tile (queries x keys) of every (batch, head): S = Q K^T and
// dP = dO V^T as 3xTF32 products (the two products' K steps one after the
// other through the stage ring, each product's accumulations summed in its own
// registers), then P = exp(S * scale - lse) and dS = P (dP - delta) * scale per
// element (zero above the diagonal), written as TF32 pairs (hi = rn(v),
// lo = rn(v - hi)): P to Ph, Pl and dS to Dh, Dl, the score buffers' layout.
struct X3ScoreMaps {
  CUtensorMap qh, ql, kh, kl, gh, gl, vh, vl;  // g: dO
};

struct X3ScoreOut {
  float *ph, *pl, *dh, *dl;
  long long ldS;
  const float* lse;    // [batch * T], the forward's log-sum-exp per query row
  const float* delta;  // [batch * T], rowsum(dO * O)
  float scale;
};

template <int BN>
__global__ void __launch_bounds__(X3_THREADS, 1)
    attn3x_scores_grad_kernel(const __grid_constant__ X3ScoreMaps maps, X3ScoreOut out, int T, int K, int* err,
                              GemmBatch bt, int total_tiles) {
  using TL = X3BatchTile<BN>;
  constexpr int STAGES = TL::STAGES;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw_addr);
  const uint32_t bar_base = base + STAGES * TL::STAGE;
  auto full_bar = [&](int s) { return bar_base + 8u * s; };
  auto empty_bar = [&](int s) { return bar_base + 8u * (STAGES + s); };
  auto acc_full = [&](int b) { return bar_base + 8u * (2 * STAGES + b); };
  auto acc_empty = [&](int b) { return bar_base + 8u * (2 * STAGES + 2 + b); };
  constexpr int kBars = 2 * STAGES + 4;
  const uint32_t tmem_slot = bar_base + 8u * kBars;
  uint8_t* tail = smem + STAGES * TL::STAGE + 8 * kBars;
  uint32_t* tmem_slot_ptr = reinterpret_cast<uint32_t*>(tail);
  int* loads_issued = reinterpret_cast<int*>(tail + 8);
  int* loads_consumed = loads_issued + 1;
  static_assert(8 * kBars + 16 <= 256, "barriers and counters fit their 256 bytes");

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&maps.qh);
    tma_prefetch_desc(&maps.ql);
    tma_prefetch_desc(&maps.kh);
    tma_prefetch_desc(&maps.kl);
    tma_prefetch_desc(&maps.gh);
    tma_prefetch_desc(&maps.gl);
    tma_prefetch_desc(&maps.vh);
    tma_prefetch_desc(&maps.vl);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(acc_full(b), 1);
      mbar_init(acc_empty(b), 8);
    }
    *loads_issued = 0;
    *loads_consumed = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 2 * BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot_ptr;
  const int n_k = (K + BK - 1) / BK;  // K steps of each product

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer: S's K steps, then dP's
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
        const TileInfo ti = tile_info<BN, true>(t, T, T, K, bt);
        if (ti.skip) continue;
        const int a_zb = ti.z / bt.a_zdiv, a_zh = (ti.z % bt.a_zdiv) / bt.a_zgroup;
        const int b_zb = ti.z / bt.b_zdiv, b_zh = (ti.z % bt.b_zdiv) / bt.b_zgroup;
        for (int i = 0; i < 2 * n_k; ++i, ++it) {
          const int s = it % STAGES, round = it / STAGES;
          if (round > 0 && !mbar_wait(empty_bar(s), (round - 1) & 1, err, kErrWaitEmpty)) {
            ok = false;
            break;
          }
          const uint32_t sa = base + s * TL::STAGE, sb = sa + 2 * TL::A_BYTES;
          mbar_arrive_expect_tx(full_bar(s), TL::STAGE);
          const bool dp = i >= n_k;
          const int k0 = (dp ? i - n_k : i) * BK;
          load_box<true>(sa, dp ? &maps.gh : &maps.qh, full_bar(s), k0, ti.m0, a_zh, a_zb);
          load_box<true>(sa + TL::A_BYTES, dp ? &maps.gl : &maps.ql, full_bar(s), k0, ti.m0, a_zh, a_zb);
          load_box<true>(sb, dp ? &maps.vh : &maps.kh, full_bar(s), k0, ti.n0, b_zh, b_zb);
          load_box<true>(sb + TL::B_BYTES, dp ? &maps.vl : &maps.kl, full_bar(s), k0, ti.n0, b_zh, b_zb);
          *loads_issued = it + 1;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- UMMA issuer: X3_CHUNK-step accumulations, none spanning the two products
      constexpr uint32_t idesc = idesc_tf32(BM, BN, false, false);
      int it = 0, j = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
        const TileInfo ti = tile_info<BN, true>(t, T, T, K, bt);
        if (ti.skip) continue;
        for (int pr = 0; pr < 2 && ok; ++pr) {
          for (int cb = 0; cb < n_k && ok; cb += X3_CHUNK) {
            const int ce = min(n_k, cb + X3_CHUNK);
            const int buf = j & 1;
            if (j >= 2 && !mbar_wait(acc_empty(buf), ((j >> 1) - 1) & 1, err, kErrWaitAccum)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t acc = tmem_base + buf * BN;
            for (int i = cb; i < ce; ++i, ++it) {
              const int s = it % STAGES, round = it / STAGES;
              if (!mbar_wait(full_bar(s), round & 1, err, kErrWaitFull)) {
                ok = false;
                break;
              }
              tc_fence_after();
              *loads_consumed = it + 1;
              const uint32_t sa = base + s * TL::STAGE, sb = sa + 2 * TL::A_BYTES;
#pragma unroll
              for (int term = 0; term < 3; ++term) {
#pragma unroll
                for (int k = 0; k < BK / 8; ++k) {
                  const uint32_t at = sa + (term == 0 ? TL::A_BYTES : 0);
                  const uint32_t bt_ = sb + (term == 1 ? TL::B_BYTES : 0);
                  umma_tf32(acc, smem_desc(at + k * 32, 16, 1024, kLayoutSw128),
                            smem_desc(bt_ + k * 32, 16, 1024, kLayoutSw128), idesc,
                            (i != cb || term != 0 || k != 0) ? 1u : 0u);
                }
              }
              umma_commit(empty_bar(s));
            }
            if (!ok) break;
            umma_commit(acc_full(buf));
            ++j;
          }
        }
      }
    }
  } else {
    // ---------------- epilogue: 32 query rows x BN / 2 keys of the tile per warp
    constexpr int NC = BN / 2;
    const int quarter = warp & 3, half = (warp - 2) >> 2;
    float4* stage_tile = reinterpret_cast<float4*>(smem + STAGES * TL::STAGE + 256) + (warp - 2) * 256;
    int j = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
      const TileInfo ti = tile_info<BN, true>(t, T, T, K, bt);
      if (ti.skip) continue;
      const int q = ti.m0 + quarter * 32 + lane, k0 = ti.n0 + half * NC;  // this thread's query row, first key
      const long long li = static_cast<long long>(ti.z) * T + q;
      const long long zoff = (ti.z / bt.c_zdiv) * bt.c_sb + ((ti.z % bt.c_zdiv) / bt.c_zgroup) * bt.c_sh;
      const int wrow0 = ti.m0 + quarter * 32;
      float pv[NC], sum[NC];
#pragma unroll
      for (int pr = 0; pr < 2; ++pr) {  // S, then dP
#pragma unroll
        for (int e = 0; e < NC; ++e) sum[e] = 0.0f;
        for (int cb = 0; ok && cb < n_k; cb += X3_CHUNK) {
          const int buf = j & 1;
          if (!mbar_wait(acc_full(buf), (j >> 1) & 1, err, kErrWaitAccum)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t acc = tmem_base + buf * BN + (static_cast<uint32_t>(quarter * 32) << 16) + half * NC;
#pragma unroll
          for (int c = 0; c < NC / 16; ++c) {
            uint32_t r[16];
            tmem_ld_32x32b_x16(acc + c * 16, r);
#pragma unroll
            for (int e = 0; e < 16; ++e) sum[c * 16 + e] += __uint_as_float(r[e]);
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(acc_empty(buf));
          ++j;
        }
        if (!ok) break;
        if (pr == 0) {  // P = exp(S * scale - lse) = 2^(S * scale log2 e - lse log2 e), written while the UMMAs form dP
          constexpr float kLog2e = 1.4426950408889634f;
          const float lse2 = q < T ? out.lse[li] * kLog2e : 0.0f, scale2 = out.scale * kLog2e;
#pragma unroll
          for (int e = 0; e < NC; ++e)
            pv[e] = (q < T && k0 + e <= q) ? ex2_approx(fmaf(sum[e], scale2, -lse2)) : 0.0f;
          store_pair<NC>(pv, stage_tile, wrow0, k0, out.ph + zoff, out.pl + zoff, out.ldS, T, T);
        } else {  // dS = P (dP - delta) * scale
          const float dl = q < T ? out.delta[li] : 0.0f;
#pragma unroll
          for (int e = 0; e < NC; ++e) sum[e] = (pv[e] * (sum[e] - dl)) * out.scale;
          store_pair<NC>(sum, stage_tile, wrow0, k0, out.dh + zoff, out.dl + zoff, out.ldS, T, T);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = *loads_consumed; i < *loads_issued; ++i)
      if (!mbar_wait(full_bar(i % STAGES), (i / STAGES) & 1, err, kErrWaitDrain, 1000000000ull)) break;
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 2 * BN);
  }
  __syncthreads();
}

}  // namespace

namespace {

// ------------------------------------------------------------------ host side

thread_local uint64_t t_launches = 0;  // kernels launched by this thread (gemm_launch_count)
thread_local cudaError_t t_launch_error = cudaSuccess;  // the last failed launch's error

// 0, or kGemmLaunch with the launch's CUDA error kept for gemm_status_string.
int launch_status() {
  const cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) return 0;
  t_launch_error = e;
  return kGemmLaunch;
}

PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// fp32 tensor map of rank 2 or 4 with a 128-byte swizzle (of 32-byte chunks for
// MN-major operands, matching the UMMA layout). dims/strides in elements;
// strides[0] is the stride of dims[1].
int encode(CUtensorMap* map, const float* ptr, int rank, const long long* dims, const long long* strides,
           const int* box, bool mn_major) {
  auto fn = get_encode_fn();
  if (!fn) return -1;
  if (rank < 2 || rank > 5) return -2;
  cuuint64_t d[5], st[4];
  cuuint32_t b[5], e[5] = {1, 1, 1, 1, 1};
  for (int i = 0; i < rank; ++i) {
    d[i] = static_cast<cuuint64_t>(dims[i]);
    b[i] = static_cast<cuuint32_t>(box[i]);
  }
  for (int i = 0; i + 1 < rank; ++i) {
    st[i] = static_cast<cuuint64_t>(strides[i]) * 4;
    if (st[i] % 16 != 0) return -2;
  }
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, rank, const_cast<float*>(ptr), d, st, b, e,
                  CU_TENSOR_MAP_INTERLEAVE_NONE,
                  mn_major ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -2;
}

}  // namespace

int encode_tensor_map(CUtensorMap* map, const float* ptr, int rank, const long long* dims, const long long* strides,
                      const int* box, bool mn_major) {
  return encode(map, ptr, rank, dims, strides, box, mn_major);
}

namespace {

// 2-D operand: `inner` contiguous elements per row, `outer` rows, `ld` apart.
int make_map2d(CUtensorMap* map, const float* ptr, long long inner, long long outer, long long ld, int box_inner,
               int box_outer, bool mn_major) {
  const long long dims[2] = {inner, outer}, strides[1] = {ld};
  const int box[2] = {box_inner, box_outer};
  return encode(map, ptr, 2, dims, strides, box, mn_major);
}

// MN-major operand (`mn` contiguous elements per K-row, rows `ld` apart) as a
// 3-D view (32 elements, K-row, 32-wide block): one box of {32, BK, box_mn / 32}
// lands as box_mn / 32 consecutive 4 KB blocks, the UMMA MN-major layout.
// Needs mn % 32 == 0 so that no block reads past a row.
int make_map_mn3d(CUtensorMap* map, const float* ptr, long long mn, long long k, long long ld, int box_mn) {
  const long long dims[3] = {32, k, mn / 32}, strides[2] = {ld, 32};
  const int box[3] = {32, BK, box_mn / 32};
  return encode(map, ptr, 3, dims, strides, box, true);
}

int device_sms() {
  static thread_local int sms = 0, sms_device = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (sms_device != dev) {
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    sms_device = dev;
  }
  return sms;
}

template <bool A_MN, bool B_MN, int BN, bool BATCHED>
void launch(const CUtensorMap& ta, const CUtensorMap& tb, float* C, long long ldc, const float* R, long long ldr,
            int M, int N, int K, int batch, const GemmBatch& bt, int* err, cudaStream_t stream, int mn3d) {
  using TL = Tile<BN>;
  auto kern = gemm_tf32_kernel<A_MN, B_MN, BN, BATCHED>;
  static thread_local int configured_device = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_device != dev) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, TL::SMEM_BYTES);
    configured_device = dev;
  }
  const long long tiles = static_cast<long long>((M + BM - 1) / BM) * ((N + BN - 1) / BN) * batch;
  const int sms = device_sms();
  const int grid = static_cast<int>(tiles < sms ? tiles : sms);
  kern<<<grid, THREADS, TL::SMEM_BYTES, stream>>>(ta, tb, C, ldc, R, ldr, M, N, K, err, bt, static_cast<int>(tiles), mn3d);
  ++t_launches;
}

template <int BN, bool BATCHED>
void launch_majors(bool a_mn, bool b_mn, const CUtensorMap& ta, const CUtensorMap& tb, float* C, long long ldc,
                   const float* R, long long ldr, int M, int N, int K, int batch, const GemmBatch& bt, int* err,
                   cudaStream_t s, int mn3d = 0) {
  if (!a_mn && !b_mn) launch<false, false, BN, BATCHED>(ta, tb, C, ldc, R, ldr, M, N, K, batch, bt, err, s, mn3d);
  else if (!a_mn && b_mn) launch<false, true, BN, BATCHED>(ta, tb, C, ldc, R, ldr, M, N, K, batch, bt, err, s, mn3d);
  else if (a_mn && !b_mn) launch<true, false, BN, BATCHED>(ta, tb, C, ldc, R, ldr, M, N, K, batch, bt, err, s, mn3d);
  else launch<true, true, BN, BATCHED>(ta, tb, C, ldc, R, ldr, M, N, K, batch, bt, err, s, mn3d);
}

// How a pair launch of `tiles` tiles on `pairs` CTA pairs cuts its last wave: the
// tiles past the last full wave are split into `splits` K parts when at least
// two parts of each fit beside one another (at most 4). Each part keeps at least
// 64 K steps (K 2,048): below that the reduce kernel costs more than the shorter
// last wave saves.
constexpr int kMinPartSteps = 64;

struct PairPlan {
  int full = 0, splits = 1;
};

PairPlan pair_plan(long long tiles, int pairs, int n_k) {
  PairPlan p;
  p.full = static_cast<int>(tiles);
  const long long tail = tiles % pairs;
  if (tail == 0) return p;
  int s = static_cast<int>(pairs / tail);
  s = s > 4 ? 4 : s;
  s = s > n_k / kMinPartSteps ? n_k / kMinPartSteps : s;
  if (s < 2) return p;
  p.full = static_cast<int>(tiles - tail);
  p.splits = s;
  return p;
}

// Workspace for split tiles: one per device (pairs x 256 KB), its uses ordered
// across streams by an event recorded after each reduce; the mutex orders the
// host side of acquire (wait on the last use) and release (record this one).
struct SplitWorkspace {
  float* ptr = nullptr;
  cudaEvent_t last_use = nullptr;
};

std::mutex& split_mutex() {
  static std::mutex mu;
  return mu;
}

SplitWorkspace* split_workspace(int dev, cudaStream_t stream, size_t floats) {
  static SplitWorkspace per_device[64];
  if (dev < 0 || dev >= 64) return nullptr;
  SplitWorkspace& w = per_device[dev];
  if (!w.ptr) {
    void* p = nullptr;
    if (cudaMalloc(&p, floats * sizeof(float)) != cudaSuccess) return nullptr;
    if (cudaEventCreateWithFlags(&w.last_use, cudaEventDisableTiming) != cudaSuccess) {
      cudaFree(p);
      return nullptr;
    }
    w.ptr = static_cast<float*>(p);
    if (cudaEventRecord(w.last_use, stream) != cudaSuccess) return nullptr;
  }
  if (cudaStreamWaitEvent(stream, w.last_use, 0) != cudaSuccess) return nullptr;
  return &w;
}

// The ticket counters of pair launches: two zeroed words per (device, stream)
// (launches on one stream run one after another, and each launch leaves its
// counter at zero). Streams past the 64th of a device get strided units.
unsigned int* unit_counter(int dev, cudaStream_t stream) {
  constexpr int kSlots = 64;
  struct Table {
    unsigned int* counters = nullptr;
    cudaStream_t streams[kSlots];
    int used = 0;
  };
  static std::mutex mu;
  static Table tables[64];
  std::lock_guard<std::mutex> lock(mu);
  if (dev < 0 || dev >= 64) return nullptr;
  Table& t = tables[dev];
  if (!t.counters) {
    void* p = nullptr;
    if (cudaMalloc(&p, kSlots * 2 * sizeof(unsigned int)) != cudaSuccess) return nullptr;
    if (cudaMemset(p, 0, kSlots * 2 * sizeof(unsigned int)) != cudaSuccess) {
      cudaFree(p);
      return nullptr;
    }
    t.counters = static_cast<unsigned int*>(p);
  }
  for (int i = 0; i < t.used; ++i)
    if (t.streams[i] == stream) return t.counters + 2 * i;
  if (t.used == kSlots) return nullptr;
  t.streams[t.used] = stream;
  return t.counters + 2 * t.used++;
}

template <bool A_MN, bool B_MN, int PN>
int launch_pair(const PairOperands& ops, float* C, long long ldc, const float* R, long long ldr, int M, int N, int* err,
                cudaStream_t stream) {
  using Cfg = PairTile<PN>;
  auto kern = gemm_pair_kernel<A_MN, B_MN, PN>;
  static thread_local int configured_device = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_device != dev) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM);
    configured_device = dev;
  }
  const int tm = (M + 2 * BM - 1) / (2 * BM);
  const long long tiles = static_cast<long long>(tm) * ((N + PN - 1) / PN);
  const int pairs = device_sms() / 2;
  const PairPlan plan = pair_plan(tiles, pairs, ops.seg_end[ops.nseg - 1]);
  const long long units = plan.full + (tiles - plan.full) * plan.splits;
  const int grid = 2 * static_cast<int>(units < pairs ? units : pairs);
  unsigned int* sched = units > pairs ? unit_counter(dev, stream) : nullptr;  // one wave needs no tickets
  if (plan.splits == 1) {
    kern<<<grid, THREADS, Cfg::SMEM, stream>>>(ops, C, ldc, R, ldr, M, N, err, static_cast<int>(tiles), plan.full, 1,
                                               nullptr, sched);
    ++t_launches;
    return 0;
  }
  std::lock_guard<std::mutex> lock(split_mutex());
  SplitWorkspace* w = split_workspace(dev, stream, static_cast<size_t>(pairs) * P_TILE_FLOATS_MAX);
  if (!w) return kGemmLaunch;
  kern<<<grid, THREADS, Cfg::SMEM, stream>>>(ops, C, ldc, R, ldr, M, N, err, static_cast<int>(tiles), plan.full,
                                             plan.splits, w->ptr, sched);
  const dim3 rgrid(static_cast<unsigned>(tiles - plan.full), 2 * BM / (256 / (PN / 4)));
  split_reduce_kernel<PN><<<rgrid, 256, 0, stream>>>(w->ptr, plan.splits, plan.full, tm, C, ldc, R, ldr, M, N);
  t_launches += 2;
  return cudaEventRecord(w->last_use, stream) == cudaSuccess ? 0 : kGemmLaunch;
}

template <int PN>
int launch_pair_majors(bool a_mn, bool b_mn, const PairOperands& ops, float* C, long long ldc, const float* R,
                       long long ldr, int M, int N, int* err, cudaStream_t s) {
  if (!a_mn && !b_mn) return launch_pair<false, false, PN>(ops, C, ldc, R, ldr, M, N, err, s);
  if (!a_mn) return launch_pair<false, true, PN>(ops, C, ldc, R, ldr, M, N, err, s);
  if (!b_mn) return launch_pair<true, false, PN>(ops, C, ldc, R, ldr, M, N, err, s);
  return launch_pair<true, true, PN>(ops, C, ldc, R, ldr, M, N, err, s);
}

template <bool A_MN, bool B_MN>
int launch_pair3x(const X3Operands& ops, float* C, long long ldc, const float* R, long long ldr, int M, int N,
                  int* err, cudaStream_t stream) {
  auto kern = gemm3x_pair_kernel<A_MN, B_MN>;
  static thread_local int configured_device = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_device != dev) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, X3_SMEM);
    configured_device = dev;
  }
  const int tm = (M + 2 * BM - 1) / (2 * BM);
  const long long tiles = static_cast<long long>(tm) * ((N + 255) / 256);
  const int pairs = device_sms() / 2;
  const PairPlan plan = pair_plan(tiles, pairs, ops.seg_end[ops.nseg - 1]);
  const long long units = plan.full + (tiles - plan.full) * plan.splits;
  const int grid = 2 * static_cast<int>(units < pairs ? units : pairs);
  if (plan.splits == 1) {
    kern<<<grid, X3_THREADS, X3_SMEM, stream>>>(ops, C, ldc, R, ldr, M, N, err, static_cast<int>(tiles), plan.full, 1,
                                                nullptr);
    ++t_launches;
    return 0;
  }
  std::lock_guard<std::mutex> lock(split_mutex());
  SplitWorkspace* w = split_workspace(dev, stream, static_cast<size_t>(pairs) * P_TILE_FLOATS_MAX);
  if (!w) return kGemmLaunch;
  kern<<<grid, X3_THREADS, X3_SMEM, stream>>>(ops, C, ldc, R, ldr, M, N, err, static_cast<int>(tiles), plan.full,
                                              plan.splits, w->ptr);
  const dim3 rgrid(static_cast<unsigned>(tiles - plan.full), 2 * BM / (256 / (256 / 4)));
  split_reduce_kernel<256><<<rgrid, 256, 0, stream>>>(w->ptr, plan.splits, plan.full, tm, C, ldc, R, ldr, M, N);
  t_launches += 2;
  return cudaEventRecord(w->last_use, stream) == cudaSuccess ? 0 : kGemmLaunch;
}

template <bool A_MN, bool B_MN, int BN>
void launch_batched3x(const X3BatchMaps& maps, float* C, long long ldc, const float* R, long long ldr, int M, int N,
                      int K, int batch, const GemmBatch& bt, int* err, cudaStream_t stream) {
  using TL = X3BatchTile<BN>;
  auto kern = gemm3x_batched_kernel<A_MN, B_MN, BN>;
  static thread_local int configured_device = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_device != dev) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, TL::SMEM);
    configured_device = dev;
  }
  const long long tiles = static_cast<long long>(batch) * ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  const int sms = device_sms();
  const int grid = static_cast<int>(tiles < sms ? tiles : sms);
  kern<<<grid, X3_THREADS, TL::SMEM, stream>>>(maps, C, ldc, R, ldr, M, N, K, err, bt, static_cast<int>(tiles));
  ++t_launches;
}

template <int BN>
void launch_batched3x_majors(bool a_mn, bool b_mn, const X3BatchMaps& maps, float* C, long long ldc, const float* R,
                             int M, int N, int K, int batch, const GemmBatch& bt, int* err, cudaStream_t s) {
  if (!a_mn && !b_mn) launch_batched3x<false, false, BN>(maps, C, ldc, R, ldc, M, N, K, batch, bt, err, s);
  else if (!a_mn) launch_batched3x<false, true, BN>(maps, C, ldc, R, ldc, M, N, K, batch, bt, err, s);
  else if (!b_mn) launch_batched3x<true, false, BN>(maps, C, ldc, R, ldc, M, N, K, batch, bt, err, s);
  else launch_batched3x<true, true, BN>(maps, C, ldc, R, ldc, M, N, K, batch, bt, err, s);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

uint64_t gemm_launch_count() { return t_launches; }

int sm_count() { return device_sms(); }

unsigned int* pair_ticket_counter(int dev, cudaStream_t stream) { return unit_counter(dev, stream); }

const char* gemm_status_string(int status) {
  switch (status) {
    case 0: return "ok";
    case kGemmBadArgument: return "bad GEMM argument (null pointer, negative size or unsupported tile)";
    case kGemmMisaligned: return "GEMM operand not 16-byte aligned or leading dimension not a multiple of 4";
    case kGemmTensorMap: return "cuTensorMapEncodeTiled is unavailable or rejected an operand";
    case kGemmLaunch: {
      static thread_local char text[160];
      std::snprintf(text, sizeof text, "GEMM kernel launch failed (%s)", cudaGetErrorString(t_launch_error));
      return text;
    }
    default: return "unknown GEMM status";
  }
}

namespace {

// Tensor maps of one operand pair. MN-major operands whose MN extent is a
// multiple of 32 load a whole stage in one 3-D box (flag bits: 1 A, 2 B);
// otherwise one 2-D box per 32-wide block (zero fill past MN). b_box: the B
// rows or columns one CTA loads per stage.
int make_maps(int M, int N, int K, const GemmOperand& A, const GemmOperand& B, int b_box, CUtensorMap* ta,
              CUtensorMap* tb, int* mn3d) {
  if ((A.ld & 3) || (B.ld & 3) || !aligned16(A.ptr) || !aligned16(B.ptr)) return kGemmMisaligned;
  const bool a3 = A.mn_major && M % 32 == 0, b3 = B.mn_major && N % 32 == 0;
  int rc = a3 ? make_map_mn3d(ta, A.ptr, M, K, A.ld, BM)
           : A.mn_major ? make_map2d(ta, A.ptr, M, K, A.ld, 32, BK, true)
                        : make_map2d(ta, A.ptr, K, M, A.ld, BK, BM, false);
  if (rc) return kGemmTensorMap;
  rc = b3 ? make_map_mn3d(tb, B.ptr, N, K, B.ld, b_box)
       : B.mn_major ? make_map2d(tb, B.ptr, N, K, B.ld, 32, BK, true)
                    : make_map2d(tb, B.ptr, K, N, B.ld, BK, b_box, false);
  if (rc) return kGemmTensorMap;
  *mn3d = (a3 ? 1 : 0) | (b3 ? 2 : 0);
  return 0;
}

// 256 x 256 tiles on CTA pairs when they fill the SMs (also once the last
// wave's tiles are cut into K parts); otherwise single CTAs.
bool pair_suits(int M, int N, int n_k) {
  if (n_k <= 0 || N <= 128) return false;
  const long long pair_tiles = static_cast<long long>((M + 2 * BM - 1) / (2 * BM)) * ((N + 255) / 256);
  const PairPlan plan = pair_plan(pair_tiles, device_sms() / 2, n_k);
  const long long units = plan.full + (pair_tiles - plan.full) * plan.splits;
  return 2 * pair_tiles >= device_sms() || 8 * units >= 3 * device_sms();
}

// One product on single CTAs: 128 x 256 tiles, or 128 x 128 ones for narrow
// outputs and for products whose 256-wide tiles would leave half of the SMs idle.
int gemm_single(int M, int N, int K, const GemmOperand& A, const GemmOperand& B, float* C, long long ldc,
                const float* R, long long ldr, int* d_err, cudaStream_t stream) {
  const long long tiles256 = static_cast<long long>((M + BM - 1) / BM) * ((N + 255) / 256);
  const int bn = (N <= 128 || 2 * tiles256 <= device_sms()) ? 128 : 256;
  CUtensorMap ta{}, tb{};
  int mn3d = 0;
  if (K > 0) {
    const int rc = make_maps(M, N, K, A, B, bn, &ta, &tb, &mn3d);
    if (rc) return rc;
  }
  const GemmBatch bt{};
  if (bn == 128)
    launch_majors<128, false>(A.mn_major, B.mn_major, ta, tb, C, ldc, R, ldr, M, N, K, 1, bt, d_err, stream, mn3d);
  else
    launch_majors<256, false>(A.mn_major, B.mn_major, ta, tb, C, ldc, R, ldr, M, N, K, 1, bt, d_err, stream, mn3d);
  return launch_status();
}

}  // namespace

int gemm_tf32_sum(int M, int N, const GemmSegment* segs, int nseg, float* C, long long ldc, const float* R,
                  long long ldr, int* d_err, cudaStream_t stream) {
  if (M < 0 || N < 0 || !C || nseg < 1 || !segs) return kGemmBadArgument;
  for (int g = 0; g < nseg; ++g)
    if (segs[g].K < 0 || (segs[g].K > 0 && (!segs[g].a.ptr || !segs[g].b.ptr))) return kGemmBadArgument;
  if (M == 0 || N == 0) return 0;
  if ((ldc & 3) || !aligned16(C) || (R && ((ldr & 3) || !aligned16(R)))) return kGemmMisaligned;
  // the segments that contribute, and whether one pair launch can sum them
  GemmSegment live[kMaxSegments];
  int n_live = 0, n_k = 0;
  bool same_majors = true;
  for (int g = 0; g < nseg; ++g) {
    if (segs[g].K == 0) continue;
    if (n_live == kMaxSegments) {
      same_majors = false;  // more than one launch holds
      break;
    }
    live[n_live] = segs[g];
    same_majors = same_majors && segs[g].a.mn_major == live[0].a.mn_major && segs[g].b.mn_major == live[0].b.mn_major;
    n_k += (segs[g].K + BK - 1) / BK;
    ++n_live;
  }
  if (n_live == 0) return gemm_single(M, N, 0, segs[0].a, segs[0].b, C, ldc, R, ldr, d_err, stream);
  if (same_majors && pair_suits(M, N, n_k)) {
    PairOperands ops{};
    int end = 0;
    for (int g = 0; g < n_live; ++g) {
      const int rc = make_maps(M, N, live[g].K, live[g].a, live[g].b, 128, &ops.a[g], &ops.b[g], &ops.mn3d[g]);
      if (rc) return rc;
      end += (live[g].K + BK - 1) / BK;
      ops.seg_end[g] = end;
    }
    ops.nseg = n_live;
    const int rc = launch_pair_majors<256>(live[0].a.mn_major, live[0].b.mn_major, ops, C, ldc, R, ldr, M, N, d_err,
                                           stream);
    if (rc) return rc;
    return launch_status();
  }
  // one launch per segment, each after the first accumulating into C
  for (int g = 0; g < nseg; ++g) {
    if (segs[g].K == 0 && g > 0) continue;
    const bool first = g == 0;
    const int rc = pair_suits(M, N, (segs[g].K + BK - 1) / BK)
                       ? gemm_tf32_sum(M, N, &segs[g], 1, C, ldc, first ? R : C, first ? ldr : ldc, d_err, stream)
                       : gemm_single(M, N, segs[g].K, segs[g].a, segs[g].b, C, ldc, first ? R : C, first ? ldr : ldc,
                                     d_err, stream);
    if (rc) return rc;
  }
  return 0;
}

bool gemm_3xtf32_pair_suits(int M, int N, int n_k) { return pair_suits(M, N, n_k); }

int gemm_3xtf32_pair_sum(int M, int N, const GemmSegment* hi, const GemmSegment* lo, int nseg, float* C,
                         long long ldc, const float* R, long long ldr, int* d_err, cudaStream_t stream) {
  if (M <= 0 || N <= 0 || !C || !hi || !lo || nseg < 1 || nseg > kMaxSegments) return kGemmBadArgument;
  if ((ldc & 3) || !aligned16(C) || (R && ((ldr & 3) || !aligned16(R)))) return kGemmMisaligned;
  X3Operands ops{};
  int end = 0;
  for (int g = 0; g < nseg; ++g) {
    const GemmSegment& h = hi[g];
    const GemmSegment& l = lo[g];
    if (h.K <= 0 || l.K != h.K || h.a.mn_major != hi[0].a.mn_major || h.b.mn_major != hi[0].b.mn_major ||
        l.a.mn_major != h.a.mn_major || l.b.mn_major != h.b.mn_major || l.a.ld != h.a.ld || l.b.ld != h.b.ld)
      return kGemmBadArgument;
    int mn3d_lo = 0;
    int rc = make_maps(M, N, h.K, h.a, h.b, 128, &ops.ah[g], &ops.bh[g], &ops.mn3d[g]);
    if (!rc) rc = make_maps(M, N, l.K, l.a, l.b, 128, &ops.al[g], &ops.bl[g], &mn3d_lo);
    if (rc) return rc;
    end += (h.K + BK - 1) / BK;
    ops.seg_end[g] = end;
  }
  ops.nseg = nseg;
  const bool a_mn = hi[0].a.mn_major, b_mn = hi[0].b.mn_major;
  int rc;
  if (!a_mn && !b_mn) rc = launch_pair3x<false, false>(ops, C, ldc, R, ldr, M, N, d_err, stream);
  else if (!a_mn) rc = launch_pair3x<false, true>(ops, C, ldc, R, ldr, M, N, d_err, stream);
  else if (!b_mn) rc = launch_pair3x<true, false>(ops, C, ldc, R, ldr, M, N, d_err, stream);
  else rc = launch_pair3x<true, true>(ops, C, ldc, R, ldr, M, N, d_err, stream);
  if (rc) return rc;
  return launch_status();
}

int gemm_tf32(int M, int N, int K, GemmOperand A, GemmOperand B, float* C, long long ldc, const float* R,
              long long ldr, int* d_err, cudaStream_t stream) {
  if (K < 0) return kGemmBadArgument;
  const GemmSegment seg{A, B, K};
  return gemm_tf32_sum(M, N, &seg, 1, C, ldc, R, ldr, d_err, stream);
}

// 4-D operand view (inner, head, row, batch) of a batched GEMM operand.
static int make_map4d(CUtensorMap* map, const BatchedOperand& o, int box_inner, int box_rows) {
  const long long dims[4] = {o.inner, o.heads, o.rows, o.batches};
  const long long strides[3] = {o.head_stride, o.row_stride, o.batch_stride};
  const int box[4] = {box_inner, 1, box_rows, 1};
  return encode(map, o.ptr, 4, dims, strides, box, o.mn_major);
}

int gemm_tf32_batched(int batch, int M, int N, int K, const BatchedOperand& A, const BatchedOperand& B, float* C,
                      long long ldc, const GemmBatch& bt_in, int bn, int* d_err, cudaStream_t stream, const float* R) {
  GemmBatch bt = bt_in;  // operand z -> (batch, head) maps come from the operands
  bt.a_zdiv = A.zdiv;
  bt.a_zgroup = A.zgroup;
  bt.b_zdiv = B.zdiv;
  bt.b_zgroup = B.zgroup;
  if (batch < 0 || M < 0 || N < 0 || K <= 0 || !C || !A.ptr || !B.ptr) return kGemmBadArgument;
  if (batch == 0 || M == 0 || N == 0) return 0;
  if (bn != 64 && bn != 128 && bn != 256) return kGemmBadArgument;
  if ((ldc & 3) || !aligned16(C) || !aligned16(A.ptr) || !aligned16(B.ptr)) return kGemmMisaligned;
  if ((bt.c_sb & 3) || (bt.c_sh & 3) || bt.a_zdiv <= 0 || bt.b_zdiv <= 0 || bt.c_zdiv <= 0 || bt.a_zgroup <= 0 ||
      bt.b_zgroup <= 0 || bt.c_zgroup <= 0 || bt.k_off < 0 || (bt.k_off % BK))
    return kGemmBadArgument;
  if (R && !aligned16(R)) return kGemmMisaligned;
  bt.skip_empty = R == C ? 1 : 0;
  CUtensorMap ta{}, tb{};
  int rc = A.mn_major ? make_map4d(&ta, A, 32, BK) : make_map4d(&ta, A, BK, BM);
  if (rc) return kGemmTensorMap;
  rc = B.mn_major ? make_map4d(&tb, B, 32, BK) : make_map4d(&tb, B, BK, bn);
  if (rc) return kGemmTensorMap;
  if (bn == 64)
    launch_majors<64, true>(A.mn_major, B.mn_major, ta, tb, C, ldc, R, ldc, M, N, K, batch, bt, d_err, stream);
  else if (bn == 128)
    launch_majors<128, true>(A.mn_major, B.mn_major, ta, tb, C, ldc, R, ldc, M, N, K, batch, bt, d_err, stream);
  else
    launch_majors<256, true>(A.mn_major, B.mn_major, ta, tb, C, ldc, R, ldc, M, N, K, batch, bt, d_err, stream);
  return launch_status();
}

int attention_scores_grad_3x(int batch, int T, int hd, const BatchedOperand& Qh, const BatchedOperand& Ql,
                             const BatchedOperand& Kh, const BatchedOperand& Kl, const BatchedOperand& Gh,
                             const BatchedOperand& Gl, const BatchedOperand& Vh, const BatchedOperand& Vl, float* Ph,
                             float* Pl, float* Dh, float* Dl, long long ldS, const GemmBatch& bt_in, const float* lse,
                             const float* delta, float scale, int* d_err, cudaStream_t stream) {
  GemmBatch bt = bt_in;
  bt.a_zdiv = Qh.zdiv;
  bt.a_zgroup = Qh.zgroup;
  bt.b_zdiv = Kh.zdiv;
  bt.b_zgroup = Kh.zgroup;
  if (batch < 0 || T < 0 || hd <= 0 || !Ph || !Pl || !Dh || !Dl || !lse || !delta) return kGemmBadArgument;
  if (batch == 0 || T == 0) return 0;
  const BatchedOperand* ops[8] = {&Qh, &Ql, &Kh, &Kl, &Gh, &Gl, &Vh, &Vl};
  for (const BatchedOperand* o : ops)
    if (!o->ptr || o->mn_major || !aligned16(o->ptr)) return o->ptr && !o->mn_major ? kGemmMisaligned : kGemmBadArgument;
  if (Gh.zdiv != Qh.zdiv || Gh.zgroup != Qh.zgroup || Vh.zdiv != Kh.zdiv || Vh.zgroup != Kh.zgroup)
    return kGemmBadArgument;  // dO is addressed like Q, V like K
  if ((ldS & 3) || !aligned16(Ph) || !aligned16(Pl) || !aligned16(Dh) || !aligned16(Dl) || (bt.c_sb & 3) ||
      (bt.c_sh & 3))
    return kGemmMisaligned;
  bt.causal = kCausalSkipUpper;
  bt.k_off = 0;
  bt.skip_empty = 0;
  constexpr int BN = 128;  // 128 x 64 tiles measured 5% slower (each UMMA then reads A for half the work)
  X3ScoreMaps maps{};
  auto map = [&](CUtensorMap* m, const BatchedOperand& o, int rows) { return make_map4d(m, o, BK, rows); };
  if (map(&maps.qh, Qh, BM) || map(&maps.ql, Ql, BM) || map(&maps.gh, Gh, BM) || map(&maps.gl, Gl, BM) ||
      map(&maps.kh, Kh, BN) || map(&maps.kl, Kl, BN) || map(&maps.vh, Vh, BN) || map(&maps.vl, Vl, BN))
    return kGemmTensorMap;
  using TL = X3BatchTile<BN>;
  auto kern = attn3x_scores_grad_kernel<BN>;
  static thread_local int configured_device = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_device != dev) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, TL::SMEM);
    configured_device = dev;
  }
  const long long tiles = static_cast<long long>(batch) * ((T + BM - 1) / BM) * ((T + BN - 1) / BN);
  const int sms = device_sms();
  const X3ScoreOut out{Ph, Pl, Dh, Dl, ldS, lse, delta, scale};
  kern<<<static_cast<int>(tiles < sms ? tiles : sms), X3_THREADS, TL::SMEM, stream>>>(maps, out, T, hd, d_err, bt,
                                                                                      static_cast<int>(tiles));
  ++t_launches;
  return launch_status();
}

int gemm_3xtf32_batched(int batch, int M, int N, int K, const BatchedOperand& Ah, const BatchedOperand& Al,
                        const BatchedOperand& Bh, const BatchedOperand& Bl, float* C, long long ldc,
                        const GemmBatch& bt_in, int bn, int* d_err, cudaStream_t stream, const float* R) {
  GemmBatch bt = bt_in;
  bt.a_zdiv = Ah.zdiv;
  bt.a_zgroup = Ah.zgroup;
  bt.b_zdiv = Bh.zdiv;
  bt.b_zgroup = Bh.zgroup;
  if (batch < 0 || M < 0 || N < 0 || K <= 0 || !C || !Ah.ptr || !Al.ptr || !Bh.ptr || !Bl.ptr) return kGemmBadArgument;
  if (batch == 0 || M == 0 || N == 0) return 0;
  if (bn != 64 && bn != 128 && bn != 256) return kGemmBadArgument;
  auto same_view = [](const BatchedOperand& a, const BatchedOperand& b) {
    return a.mn_major == b.mn_major && a.inner == b.inner && a.heads == b.heads && a.rows == b.rows &&
           a.batches == b.batches && a.head_stride == b.head_stride && a.row_stride == b.row_stride &&
           a.batch_stride == b.batch_stride && a.zdiv == b.zdiv && a.zgroup == b.zgroup;
  };
  if (!same_view(Ah, Al) || !same_view(Bh, Bl)) return kGemmBadArgument;
  if ((ldc & 3) || !aligned16(C) || !aligned16(Ah.ptr) || !aligned16(Al.ptr) || !aligned16(Bh.ptr) ||
      !aligned16(Bl.ptr))
    return kGemmMisaligned;
  if ((bt.c_sb & 3) || (bt.c_sh & 3) || bt.a_zdiv <= 0 || bt.b_zdiv <= 0 || bt.c_zdiv <= 0 || bt.a_zgroup <= 0 ||
      bt.b_zgroup <= 0 || bt.c_zgroup <= 0 || bt.k_off < 0 || (bt.k_off % BK))
    return kGemmBadArgument;
  if (R && !aligned16(R)) return kGemmMisaligned;
  bt.skip_empty = R == C ? 1 : 0;
  X3BatchMaps maps{};
  auto map_a = [&](CUtensorMap* m, const BatchedOperand& o) {
    return o.mn_major ? make_map4d(m, o, 32, BK) : make_map4d(m, o, BK, BM);
  };
  auto map_b = [&](CUtensorMap* m, const BatchedOperand& o) {
    return o.mn_major ? make_map4d(m, o, 32, BK) : make_map4d(m, o, BK, bn);
  };
  if (map_a(&maps.ah, Ah) || map_a(&maps.al, Al) || map_b(&maps.bh, Bh) || map_b(&maps.bl, Bl)) return kGemmTensorMap;
  if (bn == 64)
    launch_batched3x_majors<64>(Ah.mn_major, Bh.mn_major, maps, C, ldc, R, M, N, K, batch, bt, d_err, stream);
  else if (bn == 128)
    launch_batched3x_majors<128>(Ah.mn_major, Bh.mn_major, maps, C, ldc, R, M, N, K, batch, bt, d_err, stream);
  else
    launch_batched3x_majors<256>(Ah.mn_major, Bh.mn_major, maps, C, ldc, R, M, N, K, batch, bt, d_err, stream);
  return launch_status();
}

}  // namespace mm
