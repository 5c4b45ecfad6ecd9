// Fused causal attention forward on the tensor cores (TF32, tcgen05 + TMEM).
//
// Per block of keys:
//   S_j = Q K_j^T         tcgen05.mma, A = Q (smem), B = K_j (smem), D in TMEM
//   P_j = exp(S_j - m)    softmax warps: tcgen05.ld of their own row, online
//                         max/sum, tcgen05.st of P_j over S_j in TMEM
//   O  += P_j V_j         tcgen05.mma with A = P_j read from TMEM, B = V_j (smem)
// so the score matrix never leaves the SM. The running maximum is only moved
// (and O rescaled in TMEM) when a row's maximum grows by more than 2^8; the
// final O / l and lse = m + log(l) are exact for any maximum used consistently.
// Computes what crates/midman-nn/src/attention.rs:79-102 does (scores scaled by
// 1/sqrt(hd), -1e9 above the diagonal, softmax over keys, P V), with grouped
// key/value heads read in place rather than expanded by copy.
//
// Two forms. head_dim 64 and 128: persistent CTA pairs over 256-query tiles
// (flash_fwd_pair_kernel, below). head_dim 32: one CTA per (128-query tile,
// batch, head) with 64-key blocks (flash_fwd_kernel), 320 threads:
//   warp 0      TMA producer (one lane): Q once, then a ring of K/V stages
//   warp 1      TMEM allocator + UMMA issuer (one lane)
//   warps 2..9  two softmax warpgroups taking alternate key blocks, each with its
//               own running max/sum and O accumulator (merged at the end); warp
//               w owns TMEM lanes 32 (w % 4) .. +31, the query rows of that quarter
// TMEM columns: three S/P buffers of 64 at 0, 64, 128 (S_{j+1} is computed
// while the softmax works on S_j), then the two O accumulators.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <stdexcept>
#include <string>

#include "attention.h"
#include "gemm.h"
#include "ptx.cuh"
#include "tma.h"

namespace mm {

namespace {

constexpr int BQ = 128;    // query rows per CTA = TMEM lanes
constexpr int BKV = 64;    // keys per block
constexpr int NSBUF = 3;   // S/P buffers
constexpr int FTHREADS = 320;  // producer, UMMA issuer, two softmax warpgroups
constexpr uint32_t O_COL = NSBUF * BKV;  // 192
constexpr float kRescaleLog2 = 8.0f;    // move the running max when it grows by more than 2^8

template <int HD>
struct FlashCfg {
  static constexpr int Q_BYTES = BQ * HD * 4;
  static constexpr int K_BYTES = BKV * HD * 4;
  static constexpr int STAGE_BYTES = 2 * K_BYTES;  // K and V
  static constexpr int FIT = (200 * 1024 - Q_BYTES) / STAGE_BYTES;
  static constexpr int STAGES = FIT > 4 ? 4 : FIT;
  static constexpr int SMEM = Q_BYTES + STAGES * STAGE_BYTES + 1024 + 256 + 2048 /*group exchange*/;
  static constexpr uint32_t TMEM_COLS = O_COL + 2 * HD <= 256 ? 256 : 512;  // O of each warpgroup
  static_assert(STAGES >= 2, "flash attention needs two K/V stages");
};

struct FlashParams {
  int T, H, G, n_qt, BH;
  long long ldo;
  float scale_log2;  // softmax scale * log2(e)
  float* o;
  float* lse;
  int* err;
};

template <int HD>
__global__ void __launch_bounds__(FTHREADS, 1)
    flash_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, FlashParams p) {
  using Cfg = FlashCfg<HD>;
  constexpr int STAGES = Cfg::STAGES;
  // heaviest query tiles (most keys) are scheduled first
  const int qt = p.n_qt - 1 - static_cast<int>(blockIdx.x) / p.BH;
  const int bh = static_cast<int>(blockIdx.x) % p.BH;
  const int b = bh / p.H, h = bh % p.H, hk = h / p.G;
  const int q0 = qt * BQ;
  const int kv_end = min(p.T, q0 + BQ);
  const int n_kv = (kv_end + BKV - 1) / BKV;
  const int row0 = b * p.T;  // first token row of this sequence

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw_addr);
  const uint32_t sQ = base;
  auto sK = [&](int s) { return base + Cfg::Q_BYTES + s * Cfg::STAGE_BYTES; };
  auto sV = [&](int s) { return sK(s) + Cfg::K_BYTES; };

  const uint32_t bars = base + Cfg::Q_BYTES + STAGES * Cfg::STAGE_BYTES;
  const uint32_t q_full = bars;
  auto k_full = [&](int s) { return bars + 8u * (1 + s); };
  auto v_full = [&](int s) { return bars + 8u * (1 + STAGES + s); };
  auto kv_empty = [&](int s) { return bars + 8u * (1 + 2 * STAGES + s); };
  auto s_full = [&](int bb) { return bars + 8u * (1 + 3 * STAGES + bb); };
  auto p_full = [&](int bb) { return bars + 8u * (1 + 3 * STAGES + NSBUF + bb); };
  auto s_free = [&](int bb) { return bars + 8u * (1 + 3 * STAGES + 2 * NSBUF + bb); };
  auto o_done = [&](int g) { return bars + 8u * (1 + 3 * STAGES + 3 * NSBUF + g); };
  const uint32_t tmem_slot = bars + 8u * (3 + 3 * STAGES + 3 * NSBUF);
  uint8_t* tail = smem + (tmem_slot - base);
  uint32_t* tmem_slot_ptr = reinterpret_cast<uint32_t*>(tail);
  // K/V stages loaded by the producer and waited on by the UMMA issuer; they
  // differ only after a timed-out wait, and teardown then drains the difference.
  int* kv_issued = reinterpret_cast<int*>(tail + 8);
  int* kv_consumed = kv_issued + 1;
  int* q_pending = kv_issued + 2;

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    mbar_init(q_full, 1);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(k_full(s), 1);
      mbar_init(v_full(s), 1);
      mbar_init(kv_empty(s), 1);
    }
    for (int bb = 0; bb < NSBUF; ++bb) {
      mbar_init(s_full(bb), 1);
      mbar_init(p_full(bb), 4);  // one arrival per softmax warp
      mbar_init(s_free(bb), 1);
    }
    mbar_init(o_done(0), 1);
    mbar_init(o_done(1), 1);
    *kv_issued = 0;
    *kv_consumed = 0;
    *q_pending = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot_ptr;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer
      *q_pending = 1;
      mbar_arrive_expect_tx(q_full, Cfg::Q_BYTES);
      tma_load_3d(sQ, &tmQ, q_full, 0, row0 + q0, h * (HD / 32));
      for (int j = 0; j < n_kv; ++j) {
        const int s = j % STAGES, r = j / STAGES;
        if (r > 0 && !mbar_wait(kv_empty(s), (r - 1) & 1, p.err, kErrWaitEmpty)) break;
        // rows past this sequence's end belong to the next one (or are zero
        // fill): they are keys after every query of the tile, always masked
        mbar_arrive_expect_tx(k_full(s), Cfg::K_BYTES);
        tma_load_3d(sK(s), &tmK, k_full(s), 0, row0 + j * BKV, hk * (HD / 32));
        mbar_arrive_expect_tx(v_full(s), Cfg::K_BYTES);
        tma_load_3d(sV(s), &tmV, v_full(s), 0, row0 + j * BKV, hk * (HD / 32));
        *kv_issued = j + 1;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- UMMA issuer
      constexpr uint32_t idesc_s = idesc_tf32(BQ, BKV, false, false);  // Q K-major, K K-major
      constexpr uint32_t idesc_o = idesc_tf32(BQ, HD, false, true);    // P (TMEM), V MN-major
      bool ok = mbar_wait(q_full, 0, p.err, kErrWaitFull);
      if (ok) *q_pending = 0;
      auto issue_s = [&](int j) -> bool {
        const int s = j % STAGES, bb = j % NSBUF, u = j / NSBUF;
        if (!mbar_wait(k_full(s), (j / STAGES) & 1, p.err, kErrWaitFull)) return false;
        if (u > 0 && !mbar_wait(s_free(bb), (u - 1) & 1, p.err, kErrWaitAccum)) return false;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < HD / 8; ++kk) {
          const uint32_t off = (kk % 4) * 32u;  // 8 tf32 = 32 bytes along the 128-byte chunk
          const uint64_t a = smem_desc(sQ + (kk / 4) * (BQ * 128) + off, 16, 1024, kLayoutSw128);
          const uint64_t bd = smem_desc(sK(s) + (kk / 4) * (BKV * 128) + off, 16, 1024, kLayoutSw128);
          umma_tf32(tmem + bb * BKV, a, bd, idesc_s, kk > 0 ? 1u : 0u);
        }
        umma_commit(s_full(bb));
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; ok && j < n_kv; ++j) {
        if (j + 1 < n_kv && !issue_s(j + 1)) break;
        const int s = j % STAGES, bb = j % NSBUF;
        if (!mbar_wait(p_full(bb), (j / NSBUF) & 1, p.err, kErrWaitAccum)) break;
        if (!mbar_wait(v_full(s), (j / STAGES) & 1, p.err, kErrWaitFull)) break;
        *kv_consumed = j + 1;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < BKV / 8; ++kk) {
          // V_j: 32-wide hd blocks of BKV key rows (LBO), 8 key rows per step
          const uint64_t bd = smem_desc(sV(s) + kk * 1024, BKV * 128, 512, kLayoutSw128Base32);
          umma_tf32_ts(tmem + O_COL + (j & 1) * HD, tmem + bb * BKV + kk * 8, bd, idesc_o,
                       (j > 1 || kk > 0) ? 1u : 0u);
        }
        umma_commit(kv_empty(s));
        umma_commit(s_free(bb));
        umma_commit(o_done(j & 1));
      }
    }
  } else {
    // ---------------- softmax + epilogue. Warpgroup grp (warps 2-5, 6-9) takes
    // the key blocks j = grp mod 2 with its own running max / sum and its own
    // O accumulator; the two partial results are merged at the end.
    const int grp = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;  // query row within the tile
    const int q = q0 + row;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t o_col = O_COL + grp * HD;
    float m_run = -INFINITY, l_run = 0.0f;
    bool ok = true;
    int k = 0;  // blocks this group has processed
    for (int j = grp; j < n_kv; j += 2, ++k) {
      const int bb = j % NSBUF;
      if (!mbar_wait(s_full(bb), (j / NSBUF) & 1, p.err, kErrWaitAccum)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t r[2][32];
      tmem_ld_32x32b_x32(tmem + lane_base + bb * BKV, r[0]);
      tmem_ld_32x32b_x32(tmem + lane_base + bb * BKV + 32, r[1]);
      const int kv0 = j * BKV;
      const bool diag = kv0 + BKV - 1 > q0;  // some key of the block follows some query of the tile
      float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int c = 0; c < 2; ++c)
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          float x = __uint_as_float(r[c][i]) * p.scale_log2;
          if (diag && kv0 + c * 32 + i > q) x = -INFINITY;
          r[c][i] = __float_as_uint(x);
          mx[i & 3] = fmaxf(mx[i & 3], x);
        }
      const float m_new = fmaxf(m_run, fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])));
      if (k == 0) {
        m_run = m_new;
      } else {
        const bool need = m_new > m_run + kRescaleLog2;
        if (__any_sync(0xffffffffu, need)) {
          // this group's O holds its blocks before j once their PV is done
          if (!mbar_wait(o_done(grp), (k - 1) & 1, p.err, kErrWaitAccum)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const float alpha = need ? ex2_approx(m_run - m_new) : 1.0f;
#pragma unroll 1
          for (int c = 0; c < HD / 32; ++c) {
            uint32_t o[32];
            tmem_ld_32x32b_x32(tmem + lane_base + o_col + c * 32, o);
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st_32x32b_x32(tmem + lane_base + o_col + c * 32, o);
          }
          if (need) {
            l_run *= alpha;
            m_run = m_new;
          }
        }
      }
      // a row with every key so far masked (possible for a group's blocks past
      // the diagonal) keeps m = -inf: exponentiate against 0 so that P = 0
      const float mref = m_run == -INFINITY ? 0.0f : m_run;
      float ls[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
      for (int c = 0; c < 2; ++c)
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float e = ex2_approx(__uint_as_float(r[c][i]) - mref);
          ls[i & 3] += e;
          r[c][i] = __float_as_uint(e);
        }
      l_run += (ls[0] + ls[1]) + (ls[2] + ls[3]);
      tmem_st_32x32b_x32(tmem + lane_base + bb * BKV, r[0]);
      tmem_st_32x32b_x32(tmem + lane_base + bb * BKV + 32, r[1]);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full(bb));
    }
    if (ok && k > 0 && !mbar_wait(o_done(grp), (k - 1) & 1, p.err, kErrWaitAccum)) ok = false;
    // publish (m, l) of this group's rows, then merge with the other group's
    // after the 256 bytes of barriers and counters: [group][m | l][row]
    float* xch = reinterpret_cast<float*>(smem + Cfg::Q_BYTES + STAGES * Cfg::STAGE_BYTES + 256);
    xch[grp * 256 + row] = m_run;
    xch[grp * 256 + 128 + row] = l_run;
    tc_fence_before();
    asm volatile("bar.sync 1, 256;" ::: "memory");  // the eight softmax warps
    tc_fence_after();
    const float m_o = xch[(1 - grp) * 256 + row], l_o = xch[(1 - grp) * 256 + 128 + row];
    if (ok) {
      const float m0 = grp == 0 ? m_run : m_o, l0 = grp == 0 ? l_run : l_o;
      const float m1 = grp == 0 ? m_o : m_run, l1 = grp == 0 ? l_o : l_run;
      const float m = fmaxf(m0, m1);
      const float a0 = l0 > 0.0f ? ex2_approx(m0 - m) : 0.0f;  // a group without blocks has l = 0
      const float a1 = l1 > 0.0f ? ex2_approx(m1 - m) : 0.0f;
      const float l = (a0 > 0.0f ? l0 * a0 : 0.0f) + (a1 > 0.0f ? l1 * a1 : 0.0f);
      const float inv = 1.0f / l;
      const float w0 = a0 * inv, w1 = a1 * inv;
      float* orow = p.o + static_cast<long long>(row0 + q) * p.ldo + static_cast<long long>(h) * HD;
#pragma unroll 1
      for (int c = grp; c < HD / 32; c += 2) {  // each group writes alternate 32-column chunks
        uint32_t o0[32], o1[32];
        tmem_ld_32x32b_x32(tmem + lane_base + O_COL + c * 32, o0);
        tmem_ld_32x32b_x32(tmem + lane_base + O_COL + HD + c * 32, o1);
        if (q < p.T) {
#pragma unroll
          for (int i = 0; i < 32; i += 4) {
            float v[4];
#pragma unroll
            for (int e = 0; e < 4; ++e)
              v[e] = (a0 > 0.0f ? __uint_as_float(o0[i + e]) * w0 : 0.0f) +
                     (a1 > 0.0f ? __uint_as_float(o1[i + e]) * w1 : 0.0f);
            *reinterpret_cast<float4*>(orow + c * 32 + i) = make_float4(v[0], v[1], v[2], v[3]);
          }
        }
      }
      if (grp == 0 && q < p.T)
        p.lse[static_cast<long long>(bh) * p.T + q] = (m + log2f(l)) * 0.69314718055994531f;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) {
    // after a timed-out wait, let every TMA copy still in flight land (bounded)
    // before the CTA's shared memory is released
    if (*q_pending) mbar_wait(q_full, 0, p.err, kErrWaitDrain, 1000000000ull);
    for (int j = *kv_consumed; j < *kv_issued; ++j) {
      const int s = j % STAGES;
      if (!mbar_wait(k_full(s), (j / STAGES) & 1, p.err, kErrWaitDrain, 1000000000ull)) break;
      if (!mbar_wait(v_full(s), (j / STAGES) & 1, p.err, kErrWaitDrain, 1000000000ull)) break;
    }
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::TMEM_COLS);
  }
  __syncthreads();
}

// ------------------------------------------------------------------ CTA pairs
// Persistent: a pair per two SMs takes 256-query blocks one after another, so
// a block's Q load and first S products overlap the previous block's last
// products and epilogue, and TMEM is allocated once per pair.
// Two CTAs of a cluster share one 256-query block: CTA r holds query rows
// q0 + 128 r ... For every 128-key block each CTA loads half of K_j (64 keys)
// and half of V_j (hd / 2 columns), so the pair reads each K/V block from L2
// once where two single CTAs read it twice. The leader (rank 0) issues every
// UMMA with M = 256 (cta_group::2): S_j = Q K_j^T (N = 128 keys) and
// O += P_j V_j (N = hd, P_j read from each CTA's own TMEM). Barriers the
// UMMA issuer waits on live in the leader; the commits that release stages,
// S buffers and O reach both CTAs.
// Two UMMA issuers in the leader: warp 1 issues the S products, warp 10 the PV
// products, so a PV is queued as soon as its P is ready.
constexpr int FPAIR_THREADS = FTHREADS + 32;
constexpr int PQ = 128;   // query rows per CTA (a pair: 256)
constexpr int PKV = 128;  // keys per block = N of the S product

template <int HD>
struct PairCfg {
  static constexpr int Q_BYTES = PQ * HD * 4;
  static constexpr int K_BYTES = (PKV / 2) * HD * 4;  // this CTA's 64 keys of K_j
  static constexpr int V_BYTES = PKV * (HD / 2) * 4;  // this CTA's hd/2 columns of V_j
  static constexpr int STAGE_BYTES = K_BYTES + V_BYTES;
  static constexpr int FIT = (200 * 1024 - Q_BYTES) / STAGE_BYTES;
  static constexpr int STAGES = FIT > 4 ? 4 : FIT;
  static constexpr int STAGE_OUT = 8 * 2048;  // a 32 x 16 output staging tile per softmax warp
  static constexpr int SMEM = Q_BYTES + STAGES * STAGE_BYTES + 1024 + 512 + 2048 /*group exchange*/ + STAGE_OUT;
  static constexpr uint32_t O_COL = 2 * PKV;  // two S/P buffers, then O of each warpgroup
  static constexpr uint32_t TMEM_COLS = 512;
  static_assert(O_COL + 2 * HD <= TMEM_COLS, "TMEM budget");
  static_assert(STAGES >= 2, "two K/V stages");
};

// Barriers and shared words of the pair kernel, after the K/V stages. The
// kernel is persistent: each pair takes 256-query tiles one after another
// (its position in the grid first, then tickets), and every role counts the
// K/V blocks of all its tiles with one global index g, so that a barrier's
// phase follows from g alone: stage g % STAGES, S/P buffer and O accumulator
// g & 1 (the softmax warpgroup g & 1 takes block g).
constexpr int kFwdRing = 4;
constexpr int kFwdUnitConsumers = 1 + 2 + 16;  // peer producer, both UMMA issuers, softmax warps of both CTAs

template <int STAGES>
struct FwdBars {
  uint32_t base;
  __device__ uint32_t q_full() const { return base; }
  __device__ uint32_t q_free() const { return base + 8u; }  // the tile's S products have read Q
  __device__ uint32_t k_full(int s) const { return base + 8u * (2 + s); }
  __device__ uint32_t v_full(int s) const { return base + 8u * (2 + STAGES + s); }
  __device__ uint32_t kv_empty(int s) const { return base + 8u * (2 + 2 * STAGES + s); }
  __device__ uint32_t s_full(int bb) const { return base + 8u * (2 + 3 * STAGES + bb); }
  __device__ uint32_t p_full(int bb) const { return base + 8u * (4 + 3 * STAGES + bb); }
  __device__ uint32_t s_free(int bb) const { return base + 8u * (6 + 3 * STAGES + bb); }
  __device__ uint32_t o_done(int g) const { return base + 8u * (8 + 3 * STAGES + g); }
  __device__ uint32_t unit_full(int r) const { return base + 8u * (10 + 3 * STAGES + r); }
  __device__ uint32_t unit_empty(int r) const { return base + 8u * (10 + 3 * STAGES + kFwdRing + r); }
  __device__ uint32_t tail() const { return base + 8u * (10 + 3 * STAGES + 2 * kFwdRing); }
  __device__ void init() const {
    mbar_init(q_full(), 1);
    mbar_init(q_free(), 1);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(k_full(s), 1);
      mbar_init(v_full(s), 1);
      mbar_init(kv_empty(s), 1);
    }
    for (int bb = 0; bb < 2; ++bb) {
      mbar_init(s_full(bb), 1);
      mbar_init(p_full(bb), 8);  // four softmax warps in each CTA
      mbar_init(s_free(bb), 1);
      mbar_init(o_done(bb), 1);
    }
    for (int r = 0; r < kFwdRing; ++r) {
      mbar_init(unit_full(r), 1);
      mbar_init(unit_empty(r), kFwdUnitConsumers);
    }
  }
};

struct FwdTail {
  uint32_t tmem;
  int q_issued, q_consumed;    // Q loads issued (producer) and waited for (issuer A)
  int kv_issued, kv_consumed;  // K/V blocks loaded (producer) and read by a PV product (issuer B)
  int ring[kFwdRing];          // tile of each unit slot (-1: no more tiles)
};
static_assert(8 * (10 + 3 * 4 + 2 * kFwdRing) + sizeof(FwdTail) <= 512, "barrier area");

struct FwdTile {
  int b, h, hk, q0, n_kv;
};

__device__ __forceinline__ FwdTile fwd_tile(const FlashParams& p, int t) {
  FwdTile x;
  const int qt = p.n_qt - 1 - t / p.BH;  // heaviest 256-query blocks first
  const int bh = t % p.BH;
  x.b = bh / p.H;
  x.h = bh % p.H;
  x.hk = x.h / p.G;
  x.q0 = qt * 2 * PQ;
  x.n_kv = (min(p.T, x.q0 + 2 * PQ) + PKV - 1) / PKV;
  return x;
}

template <int HD>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(FPAIR_THREADS, 1)
    flash_fwd_pair_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                          const __grid_constant__ CUtensorMap tmV, FlashParams p, unsigned int* sched) {
  using Cfg = PairCfg<HD>;
  constexpr int STAGES = Cfg::STAGES;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = static_cast<int>(blockIdx.x) / 2, npairs = static_cast<int>(gridDim.x) / 2;
  const int n_tiles = p.n_qt * p.BH;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw_addr);
  const uint32_t sQ = base;
  auto sK = [&](int s) { return base + Cfg::Q_BYTES + s * Cfg::STAGE_BYTES; };
  auto sV = [&](int s) { return sK(s) + Cfg::K_BYTES; };
  const FwdBars<STAGES> bars{base + Cfg::Q_BYTES + STAGES * Cfg::STAGE_BYTES};
  FwdTail* tl = reinterpret_cast<FwdTail*>(smem + (bars.tail() - base));
  volatile int* ring = tl->ring;
  float* xch = reinterpret_cast<float*>(smem + Cfg::Q_BYTES + STAGES * Cfg::STAGE_BYTES + 512);
  float4* stage_out = reinterpret_cast<float4*>(smem + Cfg::Q_BYTES + STAGES * Cfg::STAGE_BYTES + 512 + 2048);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    bars.init();
    tl->q_issued = tl->q_consumed = tl->kv_issued = tl->kv_consumed = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    tmem_alloc_pair(bars.tail(), Cfg::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers initialised and TMEM allocated
  tc_fence_after();
  const uint32_t tmem = tl->tmem;

  // A consumer role's next tile (one lane): wait for the unit slot, read it,
  // free it on the leader.
  auto next_unit = [&](int& ring_i) -> int {
    const int rs = ring_i % kFwdRing, rr = ring_i / kFwdRing;
    ++ring_i;
    const bool got = leader ? mbar_wait(bars.unit_full(rs), rr & 1, p.err, kErrWaitUnit)
                            : mbar_wait_cluster(bars.unit_full(rs), rr & 1, p.err, kErrWaitUnit);
    if (!got) return -1;
    const int u = ring[rs];
    if (leader)
      mbar_arrive(bars.unit_empty(rs));
    else
      mbar_arrive_remote_release(mapa_shared(bars.unit_empty(rs), 0));
    return u;
  };

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer (both CTAs); completions land on the leader's
      // barriers. The leader takes the tiles: tickets one tile ahead; a ticket past
      // the last tile ends the pair and counts it finished, and the last pair to
      // finish resets the counter for the next launch on the stream.
      auto take_ticket = [&]() -> unsigned { return atomicAdd(&sched[0], 1u); };
      auto unit_of_ticket = [&](unsigned ticket) -> int {
        const int v = npairs + static_cast<int>(ticket);
        if (v < n_tiles) return v;
        __threadfence();
        if (atomicAdd(&sched[1], 1u) == static_cast<unsigned>(npairs - 1)) {
          __threadfence();
          atomicExch(&sched[0], 0u);
          atomicExch(&sched[1], 0u);
        }
        return -1;
      };
      int ring_i = 0, g = 0, ti = 0;
      bool ok = true;
      int u = leader ? pair : -1;
      unsigned ticket = (leader && sched) ? take_ticket() : 0u;  // the tile after u
      for (;;) {
        const int rs = ring_i % kFwdRing, rr = ring_i / kFwdRing;
        if (leader) {  // publish this tile (or the end) to the pair
          if (rr > 0 && !mbar_wait_cluster(bars.unit_empty(rs), (rr - 1) & 1, p.err, kErrWaitUnit)) {
            ok = false;
            break;
          }
          ring[rs] = u;
          st_shared_cluster(mapa_shared(smem_u32(const_cast<int*>(&ring[rs])), 1), u);
          mbar_arrive(bars.unit_full(rs));
          mbar_arrive_remote_release(mapa_shared(bars.unit_full(rs), 1));
        } else {
          if (!mbar_wait_cluster(bars.unit_full(rs), rr & 1, p.err, kErrWaitUnit)) {
            ok = false;
            break;
          }
          u = ring[rs];
          mbar_arrive_remote_release(mapa_shared(bars.unit_empty(rs), 0));
        }
        ++ring_i;
        if (u >= n_tiles) {  // never handed out
          atomicCAS(p.err, 0, kErrWaitUnit);
          u = -1;
        }
        if (u < 0) break;
        const FwdTile x = fwd_tile(p, u);
        const int row0 = x.b * p.T;
        // Q once the previous tile's S products have read theirs
        if (ti > 0 && !mbar_wait(bars.q_free(), (ti - 1) & 1, p.err, kErrWaitEmpty)) {
          ok = false;
          break;
        }
        if (leader) mbar_arrive_expect_tx(bars.q_full(), 2 * Cfg::Q_BYTES);
        tma_load_3d_pair(sQ, &tmQ, mapa_shared(bars.q_full(), 0), 0, row0 + x.q0 + static_cast<int>(rank) * PQ,
                         x.h * (HD / 32));
        tl->q_issued = ++ti;
        for (int j = 0; j < x.n_kv; ++j, ++g) {
          const int s = g % STAGES, r = g / STAGES;
          if (r > 0 && !mbar_wait(bars.kv_empty(s), (r - 1) & 1, p.err, kErrWaitEmpty)) {
            ok = false;
            break;
          }
          if (leader) {
            mbar_arrive_expect_tx(bars.k_full(s), 2 * Cfg::K_BYTES);
            mbar_arrive_expect_tx(bars.v_full(s), 2 * Cfg::V_BYTES);
          }
          // keys past this sequence's end follow every query of the pair: masked
          tma_load_3d_pair(sK(s), &tmK, mapa_shared(bars.k_full(s), 0), 0,
                           row0 + j * PKV + static_cast<int>(rank) * (PKV / 2), x.hk * (HD / 32));
          tma_load_3d_pair(sV(s), &tmV, mapa_shared(bars.v_full(s), 0), 0, row0 + j * PKV,
                           x.hk * (HD / 32) + static_cast<int>(rank) * (HD / 64));
          tl->kv_issued = g + 1;
        }
        if (!ok) break;
        if (leader) {
          if (!sched) {
            u = u + npairs < n_tiles ? u + npairs : -1;
          } else {
            u = unit_of_ticket(ticket);
            if (u >= 0) ticket = take_ticket();
          }
        }
      }
      // keep the ticket protocol whole after a timed-out wait
      if (leader && sched && u >= 0) {
        while ((u = unit_of_ticket(ticket)) >= 0) ticket = take_ticket();
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ---------------- UMMA issuer A (leader only), M = 256 across the pair: S = Q K^T
      constexpr uint32_t idesc_s = idesc_tf32(2 * PQ, PKV, false, false);
      const uint64_t dq0 = smem_desc(sQ, 16, 1024, kLayoutSw128);
      int ring_i = 0, g = 0, ti = 0;
      for (bool ok = true; ok;) {
        const int u = next_unit(ring_i);
        if (u < 0 || u >= n_tiles) break;
        const int n_kv = fwd_tile(p, u).n_kv;
        if (!mbar_wait(bars.q_full(), ti & 1, p.err, kErrWaitFull)) break;
        tl->q_consumed = ++ti;
        for (int j = 0; j < n_kv; ++j, ++g) {
          const int s = g % STAGES, bb = g & 1, uu = g >> 1;
          if (!mbar_wait(bars.k_full(s), (g / STAGES) & 1, p.err, kErrWaitFull) ||
              (uu > 0 && !mbar_wait(bars.s_free(bb), (uu - 1) & 1, p.err, kErrWaitAccum))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t dk0 = smem_desc(sK(s), 16, 1024, kLayoutSw128);
#pragma unroll
          for (int kk = 0; kk < HD / 8; ++kk) {
            const uint32_t off = (kk % 4) * 32u;  // 8 tf32 = 32 bytes along the 128-byte chunk
            umma_tf32_pair(tmem + bb * PKV, desc_add(dq0, (kk / 4) * (PQ * 128) + off),
                           desc_add(dk0, (kk / 4) * ((PKV / 2) * 128) + off), idesc_s, kk > 0 ? 1u : 0u);
          }
          umma_commit_pair(bars.s_full(bb), 0x3);
        }
        if (ok) umma_commit_pair(bars.q_free(), 0x3);
      }
    }
  } else if (warp == FTHREADS / 32) {
    if (lane == 0 && leader) {
      // ---------------- UMMA issuer B (leader only): O_{g&1} += P V once the block's
      // softmax is done; a tile's first block of each accumulator overwrites it
      constexpr uint32_t idesc_o = idesc_tf32(2 * PQ, HD, false, true);
      int ring_i = 0, g = 0;
      for (bool ok = true; ok;) {
        const int u = next_unit(ring_i);
        if (u < 0 || u >= n_tiles) break;
        const int n_kv = fwd_tile(p, u).n_kv;
        for (int j = 0; j < n_kv; ++j, ++g) {
          const int s = g % STAGES, bb = g & 1;
          if (!mbar_wait(bars.p_full(bb), (g >> 1) & 1, p.err, kErrWaitAccum) ||
              !mbar_wait(bars.v_full(s), (g / STAGES) & 1, p.err, kErrWaitFull)) {
            ok = false;
            break;
          }
          tl->kv_consumed = g + 1;
          tc_fence_after();
          // this CTA's half of V_j: 32-wide hd blocks of PKV key rows (LBO), 8 key rows per step
          const uint64_t dv0 = smem_desc(sV(s), PKV * 128, 512, kLayoutSw128Base32);
#pragma unroll
          for (int kk = 0; kk < PKV / 8; ++kk)
            umma_tf32_ts_pair(tmem + Cfg::O_COL + bb * HD, tmem + bb * PKV + kk * 8, desc_add(dv0, kk * 1024),
                              idesc_o, (j > 1 || kk > 0) ? 1u : 0u);
          umma_commit_pair(bars.kv_empty(s), 0x3);
          umma_commit_pair(bars.s_free(bb), 0x1);
          umma_commit_pair(bars.o_done(bb), 0x3);
        }
      }
    }
  } else {
    // ---------------- softmax + epilogue (both CTAs): warpgroup grp takes the
    // blocks g = grp mod 2, which use S/P buffer grp and O accumulator grp
    const int grp = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t s_col = grp * PKV;
    const uint32_t o_col = Cfg::O_COL + grp * HD;
    const uint32_t p_full_lead = mapa_shared(bars.p_full(grp), 0);
    int ring_i = 0, g0 = 0;  // g0: global index of the tile's first block
    bool ok = true;
    while (ok) {
      int u = -1;
      if (lane == 0) u = next_unit(ring_i);
      u = __shfl_sync(0xffffffffu, u, 0);
      if (u < 0 || u >= n_tiles) break;
      const FwdTile x = fwd_tile(p, u);
      const int my_q0 = x.q0 + static_cast<int>(rank) * PQ;
      const int q = my_q0 + row;
      float m_run = -INFINITY, l_run = 0.0f;
      int k = 0, last_g = 0;
      for (int j = ((g0 & 1) == grp ? 0 : 1); j < x.n_kv; j += 2, ++k) {
        const int g = g0 + j;
        if (!mbar_wait(bars.s_full(grp), (g >> 1) & 1, p.err, kErrWaitAccum)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t r[PKV];
        tmem_ld_32x32b_x128(tmem + lane_base + s_col, r);
        const int kv0 = j * PKV;
        const bool diag = kv0 + PKV - 1 > my_q0;
        float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int i = 0; i < PKV; ++i) {
          float xs = __uint_as_float(r[i]) * p.scale_log2;
          if (diag && kv0 + i > q) xs = -INFINITY;
          r[i] = __float_as_uint(xs);
          mx[i & 3] = fmaxf(mx[i & 3], xs);
        }
        const float m_new = fmaxf(m_run, fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])));
        if (k == 0) {
          m_run = m_new;
        } else {
          const bool need = m_new > m_run + kRescaleLog2;
          if (__any_sync(0xffffffffu, need)) {
            // O of this group holds the blocks up to g - 2: wait for that PV product
            if (!mbar_wait(bars.o_done(grp), ((g >> 1) - 1) & 1, p.err, kErrWaitAccum)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const float alpha = need ? ex2_approx(m_run - m_new) : 1.0f;
#pragma unroll 1
            for (int c = 0; c < HD / 32; ++c) {
              uint32_t o[32];
              tmem_ld_32x32b_x32(tmem + lane_base + o_col + c * 32, o);
#pragma unroll
              for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
              tmem_st_32x32b_x32(tmem + lane_base + o_col + c * 32, o);
            }
            if (need) {
              l_run *= alpha;
              m_run = m_new;
            }
          }
        }
        const float mref = m_run == -INFINITY ? 0.0f : m_run;
        float ls[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int i = 0; i < PKV; ++i) {
          const float e = ex2_approx(__uint_as_float(r[i]) - mref);
          ls[i & 3] += e;
          r[i] = __float_as_uint(e);
        }
        l_run += (ls[0] + ls[1]) + (ls[2] + ls[3]);
        tmem_st_32x32b_x128(tmem + lane_base + s_col, r);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(p_full_lead);
        last_g = g;
      }
      g0 += x.n_kv;
      if (ok && k > 0 && !mbar_wait(bars.o_done(grp), (last_g >> 1) & 1, p.err, kErrWaitAccum)) ok = false;
      xch[grp * 256 + row] = m_run;
      xch[grp * 256 + 128 + row] = l_run;
      tc_fence_before();
      asm volatile("bar.sync 1, 256;" ::: "memory");  // the eight softmax warps of this CTA
      tc_fence_after();
      const float m_o = xch[(1 - grp) * 256 + row], l_o = xch[(1 - grp) * 256 + 128 + row];
      if (ok) {
        const float m0 = grp == 0 ? m_run : m_o, l0 = grp == 0 ? l_run : l_o;
        const float m1 = grp == 0 ? m_o : m_run, l1 = grp == 0 ? l_o : l_run;
        const float m = fmaxf(m0, m1);
        const float a0 = l0 > 0.0f ? ex2_approx(m0 - m) : 0.0f;
        const float a1 = l1 > 0.0f ? ex2_approx(m1 - m) : 0.0f;
        const float l = (a0 > 0.0f ? l0 * a0 : 0.0f) + (a1 > 0.0f ? l1 * a1 : 0.0f);
        const float inv = 1.0f / l;
        const float w0 = a0 * inv, w1 = a1 * inv;
        // Rows leave through this warp's staging tile, 16 columns at a time
        // (4-float granules XOR-swizzled by row), so that each store
        // instruction writes eight whole 64-byte row segments.
        float4* wst = stage_out + (warp - 2) * 128;
        const int sub = lane & 3, rsub = lane >> 2;
        float* obase = p.o + static_cast<long long>(x.b * p.T) * p.ldo + static_cast<long long>(x.h) * HD;
#pragma unroll 1
        for (int c = grp; c < HD / 32; c += 2) {
          uint32_t o0[32], o1[32];
          tmem_ld_32x32b_x32(tmem + lane_base + Cfg::O_COL + c * 32, o0);
          tmem_ld_32x32b_x32(tmem + lane_base + Cfg::O_COL + HD + c * 32, o1);
#pragma unroll
          for (int half = 0; half < 2; ++half) {
#pragma unroll
            for (int gr = 0; gr < 4; ++gr) {
              float v[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const int i = half * 16 + gr * 4 + e;
                v[e] = (a0 > 0.0f ? __uint_as_float(o0[i]) * w0 : 0.0f) +
                       (a1 > 0.0f ? __uint_as_float(o1[i]) * w1 : 0.0f);
              }
              wst[lane * 4 + (gr ^ (lane & 3))] = make_float4(v[0], v[1], v[2], v[3]);
            }
            __syncwarp();
#pragma unroll
            for (int it = 0; it < 4; ++it) {
              const int rr = it * 8 + rsub;
              const float4 v = wst[rr * 4 + (sub ^ (rr & 3))];
              const int qr = my_q0 + quarter * 32 + rr;
              if (qr < p.T)
                *reinterpret_cast<float4*>(obase + static_cast<long long>(qr) * p.ldo + c * 32 + half * 16 + sub * 4) =
                    v;
            }
            __syncwarp();
          }
        }
        if (grp == 0 && q < p.T)
          p.lse[static_cast<long long>(x.b * p.H + x.h) * p.T + q] = (m + log2f(l)) * 0.69314718055994531f;
      }
      // both groups of this CTA have read O (and xch) before either group's next
      // P is published, i.e. before the next tile's PV products write O
      tc_fence_before();
      asm volatile("bar.sync 1, 256;" ::: "memory");
    }
  }

  tc_fence_before();
  cluster_sync();  // both CTAs are done with their TMEM and with each other's barriers
  if (leader && threadIdx.x == 0) {
    // after a timed-out wait, let every TMA copy of the pair still in flight
    // land (bounded) before either CTA's shared memory is released
    if (tl->q_issued > tl->q_consumed)
      mbar_wait(bars.q_full(), (tl->q_issued - 1) & 1, p.err, kErrWaitDrain, 1000000000ull);
    for (int j = tl->kv_consumed; j < tl->kv_issued; ++j) {
      const int s = j % STAGES;
      if (!mbar_wait(bars.k_full(s), (j / STAGES) & 1, p.err, kErrWaitDrain, 1000000000ull)) break;
      if (!mbar_wait(bars.v_full(s), (j / STAGES) & 1, p.err, kErrWaitDrain, 1000000000ull)) break;
    }
  }
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, Cfg::TMEM_COLS);
  }
}

bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

// Token-major operand [rows, ld] whose head `hh` occupies columns hh*HD ..: a
// 3-D view (32 columns, token row, 32-column block) so one box brings a whole
// row tile of one head, laid out as hd/32 consecutive 128-byte-wide chunks.
void head_map(CUtensorMap* map, const float* ptr, long long rows, long long ld, int heads, int hd, int box_rows,
              bool mn_major) {
  const long long dims[3] = {32, rows, static_cast<long long>(heads) * hd / 32};
  const long long strides[2] = {ld, 32};
  const int box[3] = {32, box_rows, hd / 32};
  if (encode_tensor_map(map, ptr, 3, dims, strides, box, mn_major))
    throw std::runtime_error("flash attention: tensor map rejected");
}

template <int HD>
void launch_flash(const AttnShape& s, const float* q, const float* k, const float* v, float* o, float* lse,
                  int* d_err, cudaStream_t stream) {
  using Cfg = FlashCfg<HD>;
  const long long rows = static_cast<long long>(s.B) * s.T;
  CUtensorMap tq, tk, tv;
  head_map(&tq, q, rows, s.ldq, s.H, HD, BQ, false);
  head_map(&tk, k, rows, s.ldk, s.Hkv, HD, BKV, false);
  head_map(&tv, v, rows, s.ldv, s.Hkv, HD, BKV, true);
  static thread_local int configured = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured != dev) {
    cudaFuncSetAttribute(flash_fwd_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM);
    configured = dev;
  }
  FlashParams p;
  p.T = s.T;
  p.H = s.H;
  p.G = s.H / s.Hkv;
  p.n_qt = (s.T + BQ - 1) / BQ;
  p.BH = s.B * s.H;
  p.ldo = s.ldo;
  p.scale_log2 = s.scale * 1.4426950408889634f;
  p.o = o;
  p.lse = lse;
  p.err = d_err;
  const long long grid = static_cast<long long>(p.n_qt) * p.BH;
  flash_fwd_kernel<HD><<<static_cast<unsigned>(grid), FTHREADS, Cfg::SMEM, stream>>>(tq, tk, tv, p);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string("flash attention launch: ") + cudaGetErrorString(e));
}

template <int HD>
void launch_flash_pair(const AttnShape& s, const float* q, const float* k, const float* v, float* o, float* lse,
                       int* d_err, cudaStream_t stream) {
  using Cfg = PairCfg<HD>;
  const long long rows = static_cast<long long>(s.B) * s.T;
  CUtensorMap tq, tk, tv;
  head_map(&tq, q, rows, s.ldq, s.H, HD, PQ, false);
  head_map(&tk, k, rows, s.ldk, s.Hkv, HD, PKV / 2, false);
  {  // V: each CTA of a pair takes hd/2 columns of all PKV keys
    const long long dims[3] = {32, rows, static_cast<long long>(s.Hkv) * HD / 32};
    const long long strides[2] = {s.ldv, 32};
    const int box[3] = {32, PKV, HD / 64};
    if (encode_tensor_map(&tv, v, 3, dims, strides, box, true))
      throw std::runtime_error("flash attention: tensor map rejected");
  }
  const cudaError_t a =
      cudaFuncSetAttribute(flash_fwd_pair_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM);
  if (a != cudaSuccess) throw std::runtime_error(std::string("flash attention smem: ") + cudaGetErrorString(a));
  FlashParams p;
  p.T = s.T;
  p.H = s.H;
  p.G = s.H / s.Hkv;
  p.n_qt = (s.T + 2 * PQ - 1) / (2 * PQ);
  p.BH = s.B * s.H;
  p.ldo = s.ldo;
  p.scale_log2 = s.scale * 1.4426950408889634f;
  p.o = o;
  p.lse = lse;
  p.err = d_err;
  // persistent: one pair per two SMs (fewer when there are fewer tiles); tiles
  // past the first wave go to the pairs that finish first (ticket counter)
  const long long tiles = static_cast<long long>(p.n_qt) * p.BH;
  const long long pairs = tiles < sm_count() / 2 ? tiles : sm_count() / 2;
  unsigned int* sched = nullptr;
  if (tiles > pairs) {
    int dev = 0;
    cudaGetDevice(&dev);
    sched = pair_ticket_counter(dev, stream);  // null: the pairs stride over the tiles
  }
  flash_fwd_pair_kernel<HD><<<static_cast<unsigned>(2 * pairs), FPAIR_THREADS, Cfg::SMEM, stream>>>(tq, tk, tv, p,
                                                                                                     sched);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string("flash attention launch: ") + cudaGetErrorString(e));
}

}  // namespace

bool attention_flash_supported(const AttnShape& s) {
  return (s.hd == 32 || s.hd == 64 || s.hd == 128) && s.ldq % 4 == 0 && s.ldk % 4 == 0 && s.ldv % 4 == 0 &&
         s.ldo % 4 == 0;
}

void attention_forward_flash(const AttnShape& s, const float* q, const float* k, const float* v, float* o,
                             float* lse, int* d_err, cudaStream_t stream) {
  if (!attention_flash_supported(s) || !aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o))
    throw std::runtime_error("flash attention: unsupported head_dim, stride or alignment");
  switch (s.hd) {
    case 32: launch_flash<32>(s, q, k, v, o, lse, d_err, stream); break;
    case 64: launch_flash_pair<64>(s, q, k, v, o, lse, d_err, stream); break;
    default: launch_flash_pair<128>(s, q, k, v, o, lse, d_err, stream); break;
  }
}

}  // namespace mm
