// Split-K weight-streaming GEMM on 5th-generation tensor cores (sm_100a).
//
//   part[s][n][m] = sum_{k in split s} W[m][k] * X[n][k]
//
// W is a bf16 weight [Mw, K] (row-major, K contiguous); X is the bf16 lane
// activation [2 * Ncap, K] holding a (hi, lo) row pair per lane, starting at
// row x_row0. Weight rows fill the 128-row M side of tcgen05.mma and
// decode lanes sit on N (16..256), so a handful of lanes still uses the full
// tensor-core M width. Each CTA owns one 128-row tile, one K split and one
// N tile; TMA streams 128x64 weight boxes and BNx64 activation boxes into a
// ST-deep shared-memory ring (128-byte swizzle); one thread issues the MMAs
// into a TMEM accumulator; four warps read it back with tcgen05.ld and write
// fp32 partials. The K split boundaries depend only on (K, splits), never on
// the batch, so a lane's output is bit-identical whatever batch it is in; the
// consumer sums the partials in split order.
#pragma once

#include "common.cuh"

namespace ls {

constexpr int kGemmBM = 128;
constexpr int kGemmBK = 64;   // 64 bf16 = 128 bytes = one swizzle row
constexpr int kGemmThreads = 128;

template <int BN, int ST>
struct GemmSmem {
  static constexpr int kABytes = kGemmBM * kGemmBK * 2;
  static constexpr int kBBytes = BN * kGemmBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kBarOffset = ST * kStageBytes;
  static constexpr int kTotal = 1024 /*alignment slack*/ + kBarOffset + (2 * ST + 1) * 8 + 16;
  static constexpr uint32_t kTmemCols = BN < 32 ? 32 : BN;
};

template <int BN, int ST>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                   float* __restrict__ part, int Mw, int K, int n_valid, int x_row0,
                   int splits, long split_stride, int* err) {
  using L = GemmSmem<BN, ST>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * ST + 1);
  const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + ST), acc_bar = smem_u32(bars + 2 * ST);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * kGemmBM;
  const int split = blockIdx.y;
  const int n0 = blockIdx.z * BN;
  const int KB = (K + kGemmBK - 1) / kGemmBK;
  const int kb0 = (int)((long)split * KB / splits);
  const int kb1 = (int)((long)(split + 1) * KB / splits);
  const int nkb = kb1 - kb0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < ST; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    mbar_init(acc_bar, 1);
    fence_barrier_init();
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmX);
  }
  if (warp == 2) {
    tmem_alloc(smem_u32(tmem_slot), L::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // Weights do not depend on the previous kernel: issue the first ring of
  // weight loads before waiting on it, then the activation loads after.
  if (warp == 0 && lane == 0) {
    const int pre = nkb < ST ? nkb : ST;
    for (int i = 0; i < pre; ++i) {
      const uint32_t fb = full0 + 8 * i;
      mbar_expect_tx(fb, L::kStageBytes);
      tma_load_2d(smem_u32(smem + i * L::kStageBytes), &tmW, fb, (kb0 + i) * kGemmBK, m0);
    }
    pdl_wait();
    for (int i = 0; i < pre; ++i) {
      tma_load_2d(smem_u32(smem + i * L::kStageBytes + L::kABytes), &tmX, full0 + 8 * i,
                  (kb0 + i) * kGemmBK, x_row0 + n0);
    }
    for (int i = pre; i < nkb; ++i) {
      const int s = i % ST;
      const uint32_t ph = (uint32_t)((i / ST) & 1);
      if (!mbar_wait(empty0 + 8 * s, ph ^ 1u, err, kDevTimeoutEmpty)) break;
      const uint32_t fb = full0 + 8 * s;
      mbar_expect_tx(fb, L::kStageBytes);
      uint8_t* st = smem + s * L::kStageBytes;
      tma_load_2d(smem_u32(st), &tmW, fb, (kb0 + i) * kGemmBK, m0);
      tma_load_2d(smem_u32(st + L::kABytes), &tmX, fb, (kb0 + i) * kGemmBK, x_row0 + n0);
    }
  } else if (warp == 1 && lane == 0) {
    constexpr uint32_t idesc = umma_idesc_bf16(kGemmBM, BN);
    for (int i = 0; i < nkb; ++i) {
      const int s = i % ST;
      const uint32_t ph = (uint32_t)((i / ST) & 1);
      if (!mbar_wait(full0 + 8 * s, ph, err, kDevTimeoutFull)) break;
      tc_fence_after();
      const uint32_t a = smem_u32(smem + s * L::kStageBytes);
      const uint32_t b = a + L::kABytes;
#pragma unroll
      for (int k = 0; k < kGemmBK / 16; ++k) {
        tc_mma_bf16(tmem, umma_desc_sw128(a + 32 * k), umma_desc_sw128(b + 32 * k), idesc,
                    (i | k) != 0);
      }
      tc_commit(empty0 + 8 * s);
    }
    tc_commit(acc_bar);
  }
  __syncthreads();

  // Epilogue: TMEM lane = weight row, TMEM column = activation row. Each lane
  // n owns two activation rows, 2n = bf16(x) and 2n+1 = bf16(x - bf16(x)), so
  // its output is the sum of two adjacent accumulator columns: activations
  // enter at ~16 mantissa bits for the price of idle tensor-core work only.
  const bool have = mbar_wait(acc_bar, 0, err, kDevTimeoutAcc);
  tc_fence_after();
  const int row = m0 + warp * 32 + lane;
  float* out = part + (long)split * split_stride;
#pragma unroll 1
  for (int c0 = 0; c0 < BN; c0 += 8) {
    if (n0 + c0 >= 2 * n_valid) break;
    uint32_t r[8];
    tmem_ld_32x32b_x8(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0, r);
    tmem_ld_wait();
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = (n0 + c0) / 2 + j;
      if (n < n_valid && row < Mw) {
        const float v = __uint_as_float(r[2 * j]) + __uint_as_float(r[2 * j + 1]);
        out[(long)n * Mw + row] = (have && nkb > 0) ? v : 0.f;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  pdl_launch_dependents();
  if (warp == 2) tmem_dealloc(tmem, L::kTmemCols);
}

}  // namespace ls
