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
// Warp roles (192 threads, one CTA per 128 x 256 output tile):
//   warp 0      TMA producer (one lane), STAGES-deep ring of A/B stages
//   warp 1      TMEM allocator + UMMA issuer (one lane)
//   warps 2..5  epilogue: TMEM -> registers -> global (optionally + R)
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdint>
#include <cstdio>
#include <mutex>

#include "gemm.h"
#include "ptx.cuh"

namespace mm {

namespace {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 32;  // 32 fp32 = 128 bytes = one swizzle row
constexpr int STAGES = 4;
constexpr int A_STAGE_BYTES = BM * BK * 4;  // 16 KB
constexpr int B_STAGE_BYTES = BN * BK * 4;  // 32 KB
constexpr int STAGE_BYTES = A_STAGE_BYTES + B_STAGE_BYTES;
constexpr int TMEM_COLS = 256;
constexpr int THREADS = 192;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers, TMEM slot, counters*/;

// Byte offset of the 4 KB block that holds MN columns [32j, 32j+32) of an
// MN-major tile; its 32 K-rows sit 128 bytes apart.
constexpr uint32_t MN_BLOCK_BYTES = BK * 128;

template <bool A_MN, bool B_MN>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_tf32_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     float* C, long long ldc, const float* R, long long ldr, int M,
                     int N, int K, int* err) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;  // SW128 atoms want 1024-byte alignment
  uint8_t* smem = smem_raw + (base - raw_addr);

  const uint32_t bar_base = base + STAGES * STAGE_BYTES;
  auto full_bar = [&](int s) { return bar_base + 8u * s; };
  auto empty_bar = [&](int s) { return bar_base + 8u * (STAGES + s); };
  const uint32_t accum_bar = bar_base + 8u * (2 * STAGES);
  const uint32_t tmem_slot = bar_base + 8u * (2 * STAGES + 1);
  uint32_t* tmem_slot_ptr = reinterpret_cast<uint32_t*>(smem + STAGES * STAGE_BYTES + 8 * (2 * STAGES + 1));
  // Stages loaded by the producer and consumed by the UMMA issuer; they differ
  // only when a wait timed out, and teardown then drains the difference.
  int* loads_issued = reinterpret_cast<int*>(smem + STAGES * STAGE_BYTES + 8 * (2 * STAGES + 2));
  int* loads_consumed = loads_issued + 1;

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int m0 = blockIdx.y * BM;
  const int n0 = blockIdx.x * BN;
  const int k_tiles = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    mbar_init(accum_bar, 1);
    *loads_issued = 0;
    *loads_consumed = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_acc = *tmem_slot_ptr;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer
      for (int kt = 0; kt < k_tiles; ++kt) {
        const int s = kt % STAGES;
        const int round = kt / STAGES;
        if (round > 0 && !mbar_wait(empty_bar(s), (round - 1) & 1, err, kErrWaitEmpty)) break;
        const uint32_t sa = base + s * STAGE_BYTES;
        const uint32_t sb = sa + A_STAGE_BYTES;
        mbar_arrive_expect_tx(full_bar(s), STAGE_BYTES);
        const int k0 = kt * BK;
        if (!A_MN) {
          tma_load_2d(sa, &tmA, full_bar(s), k0, m0);
        } else {
#pragma unroll
          for (int j = 0; j < BM / 32; ++j) tma_load_2d(sa + j * MN_BLOCK_BYTES, &tmA, full_bar(s), m0 + 32 * j, k0);
        }
        if (!B_MN) {
          tma_load_2d(sb, &tmB, full_bar(s), k0, n0);
        } else {
#pragma unroll
          for (int j = 0; j < BN / 32; ++j) tma_load_2d(sb + j * MN_BLOCK_BYTES, &tmB, full_bar(s), n0 + 32 * j, k0);
        }
        *loads_issued = kt + 1;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- UMMA issuer
      constexpr uint32_t idesc = idesc_tf32(BM, BN, A_MN, B_MN);
      bool ok = true;
      for (int kt = 0; kt < k_tiles && ok; ++kt) {
        const int s = kt % STAGES;
        const int round = kt / STAGES;
        ok = mbar_wait(full_bar(s), round & 1, err, kErrWaitFull);
        if (!ok) break;
        tc_fence_after();
        *loads_consumed = kt + 1;
        const uint32_t sa = base + s * STAGE_BYTES;
        const uint32_t sb = sa + A_STAGE_BYTES;
#pragma unroll
        for (int k = 0; k < BK / 8; ++k) {
          // K-major: step 8 tf32 = 32 bytes along the swizzled row.
          // MN-major: step 8 K-rows = 1024 bytes.
          // MN-major (32-byte swizzle atoms of 4 K-rows): LBO = next 32-wide MN block,
          // SBO = next group of 4 K-rows (512 bytes).
          const uint64_t adesc = A_MN ? smem_desc(sa + k * 1024, MN_BLOCK_BYTES, 512, kLayoutSw128Base32)
                                      : smem_desc(sa + k * 32, 16, 1024, kLayoutSw128);
          const uint64_t bdesc = B_MN ? smem_desc(sb + k * 1024, MN_BLOCK_BYTES, 512, kLayoutSw128Base32)
                                      : smem_desc(sb + k * 32, 16, 1024, kLayoutSw128);
          umma_tf32(tmem_acc, adesc, bdesc, idesc, (kt | k) != 0 ? 1u : 0u);
        }
        umma_commit(empty_bar(s));
      }
      umma_commit(accum_bar);
    }
  } else {
    // ---------------- epilogue: warps 2..5 cover TMEM lane quarters (warp % 4)
    const int quarter = warp & 3;
    const int row = m0 + quarter * 32 + lane;
    const bool ok = mbar_wait(accum_bar, 0, err, kErrWaitAccum);
    tc_fence_after();
    if (ok && k_tiles > 0) {
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_acc + (static_cast<uint32_t>(quarter * 32) << 16) + c * 32, r);
        const int col0 = n0 + c * 32;
        if (row < M && col0 < N) {
          float* crow = C + static_cast<long long>(row) * ldc;
          const float* rrow = R ? R + static_cast<long long>(row) * ldr : nullptr;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int col = col0 + 4 * j;
            float4 v = make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                                   __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
            if (col + 3 < N) {
              if (rrow) {
                const float4 a = *reinterpret_cast<const float4*>(rrow + col);
                v.x += a.x; v.y += a.y; v.z += a.z; v.w += a.w;
              }
              *reinterpret_cast<float4*>(crow + col) = v;
            } else {
              const float vv[4] = {v.x, v.y, v.z, v.w};
              for (int e = 0; e < 4 && col + e < N; ++e)
                crow[col + e] = vv[e] + (rrow ? rrow[col + e] : 0.0f);
            }
          }
        }
      }
    } else if (k_tiles == 0 && row < M) {
      // K == 0: the product is empty, C = R (or 0).
      for (int col = n0; col < n0 + BN && col < N; ++col)
        C[static_cast<long long>(row) * ldc + col] = R ? R[static_cast<long long>(row) * ldr + col] : 0.0f;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) {
    // Only after a timed-out wait can a TMA stage still be in flight here: let
    // each one land (bounded) before the CTA's shared memory is released.
    for (int kt = *loads_consumed; kt < *loads_issued; ++kt)
      if (!mbar_wait(full_bar(kt % STAGES), (kt / STAGES) & 1, err, kErrWaitDrain, 1000000000ull)) break;
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_acc, TMEM_COLS);
  }
  __syncthreads();
}

// ------------------------------------------------------------------ host side

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

// 2-D fp32 tensor map: `inner` contiguous elements per row, `outer` rows,
// `ld` elements between rows; box of box_inner x box_outer, 128-byte swizzle
// (of 32-byte chunks for MN-major operands, matching the UMMA layout).
int make_map(CUtensorMap* map, const float* ptr, long long inner, long long outer, long long ld,
             int box_inner, int box_outer, bool mn_major) {
  auto encode = get_encode_fn();
  if (!encode) return -1;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 4};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_inner), static_cast<cuuint32_t>(box_outer)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(ptr), dims, strides,
                      box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                      mn_major ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -2;
}

template <bool A_MN, bool B_MN>
void launch(const CUtensorMap& ta, const CUtensorMap& tb, float* C, long long ldc, const float* R,
            long long ldr, int M, int N, int K, int* err, cudaStream_t stream) {
  auto kern = gemm_tf32_kernel<A_MN, B_MN>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
  dim3 grid((N + BN - 1) / BN, (M + BM - 1) / BM);
  kern<<<grid, THREADS, SMEM_BYTES, stream>>>(ta, tb, C, ldc, R, ldr, M, N, K, err);
}

}  // namespace

const char* gemm_status_string(int status) {
  switch (status) {
    case 0: return "ok";
    case kGemmBadArgument: return "bad GEMM argument (null pointer or negative size)";
    case kGemmMisaligned: return "GEMM operand not 16-byte aligned or leading dimension not a multiple of 4";
    case kGemmTensorMap: return "cuTensorMapEncodeTiled is unavailable or rejected an operand";
    case kGemmLaunch: return "GEMM kernel launch failed";
    default: return "unknown GEMM status";
  }
}

int gemm_tf32(int M, int N, int K, GemmOperand A, GemmOperand B, float* C, long long ldc,
              const float* R, long long ldr, int* d_err, cudaStream_t stream) {
  if (M < 0 || N < 0 || K < 0 || !C) return kGemmBadArgument;
  if (M == 0 || N == 0) return 0;
  if (K > 0 && (!A.ptr || !B.ptr)) return kGemmBadArgument;
  auto aligned = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  if ((ldc & 3) || !aligned(C) || (R && ((ldr & 3) || !aligned(R)))) return kGemmMisaligned;
  CUtensorMap ta{}, tb{};
  if (K > 0) {
    if ((A.ld & 3) || (B.ld & 3) || !aligned(A.ptr) || !aligned(B.ptr)) return kGemmMisaligned;
    int rc = A.mn_major ? make_map(&ta, A.ptr, M, K, A.ld, 32, BK, true) : make_map(&ta, A.ptr, K, M, A.ld, BK, BM, false);
    if (rc) return kGemmTensorMap;
    rc = B.mn_major ? make_map(&tb, B.ptr, N, K, B.ld, 32, BK, true) : make_map(&tb, B.ptr, K, N, B.ld, BK, BN, false);
    if (rc) return kGemmTensorMap;
  }
  if (!A.mn_major && !B.mn_major) launch<false, false>(ta, tb, C, ldc, R, ldr, M, N, K, d_err, stream);
  else if (!A.mn_major && B.mn_major) launch<false, true>(ta, tb, C, ldc, R, ldr, M, N, K, d_err, stream);
  else if (A.mn_major && !B.mn_major) launch<true, false>(ta, tb, C, ldc, R, ldr, M, N, K, d_err, stream);
  else launch<true, true>(ta, tb, C, ldc, R, ldr, M, N, K, d_err, stream);
  return cudaGetLastError() == cudaSuccess ? 0 : kGemmLaunch;
}

}  // namespace mm
