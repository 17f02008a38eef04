// Weight-streaming GEMM on 5th-generation tensor cores (sm_100a) with an
// in-cluster split-K reduction and fused epilogues.
//
//   y[n][m] = sum_k W[m][k] * x[n][k]
//
// W is a bf16 weight [Mw, K] (row-major, K contiguous); x is the lane
// activation, stored as a bf16 (hi, lo) row pair per lane in X [2*Ncap, K]
// starting at row x_row0. Weight rows fill the 128-row M side of
// tcgen05.mma and activation rows sit on N (16..256), so a handful of decode
// lanes still uses the full tensor-core M width.
//
// Grid (m_tiles, splits, n_tiles), cluster (1, splits, 1): the `splits` CTAs
// of one m-tile each stream a fixed K range (boundaries depend only on K and
// splits, never on the batch). TMA streams 128x64 weight boxes and BNx64
// activation boxes into an ST-deep shared-memory ring (128-byte swizzle); one
// thread issues the MMAs into a TMEM accumulator; four warps read it back,
// add each lane's hi/lo columns and park the partial tile in shared memory.
// After a cluster barrier every CTA of the cluster reduces a slice of the
// tile's rows over all splits in split order through distributed shared
// memory, then applies the epilogue:
//   kEpiStore   y -> fp32 out[n][m]
//   kEpiQkvRope q/k rows get neox RoPE at the lane's position; k and v go to
//               the layer's KV pool at the lane's slot (bf16), q to fp32
//   kEpiSwiGLU  the tile holds 64 gate rows and their 64 up rows (two TMA
//               boxes); writes silu(g) * u as the next GEMM's (hi, lo) input
// A lane's result therefore never depends on the batch it runs in.
#pragma once

#include "common.cuh"

namespace ls {

constexpr int kGemmBM = 128;
constexpr int kGemmBK = 64;   // 64 bf16 = 128 bytes = one swizzle row
constexpr int kGemmThreads = 128;
constexpr int kMaxSplits = 8; // portable cluster size

enum GemmEpiKind : int { kEpiStore = 0, kEpiQkvRope = 1, kEpiSwiGLU = 2 };

struct GemmEpi {
  float* out;                 // store: out[n * Mw + m]
  const int* meta;            // qkv: lane metadata (int32 [cap][8], pos at 1, slot at 3)
  const float* inv_freq;      // qkv: [hd/2]
  float* q;                   // qkv: [cap][nh*hd]
  __nv_bfloat16* kpool;       // qkv: this layer's [slots][nkv*hd]
  __nv_bfloat16* vpool;
  int hd, nh, nkv, n_slots;
  __nv_bfloat16* x_act;       // swiglu: (hi, lo) rows [2*cap][I]
  int I;
};

template <int BN, int ST>
struct GemmSmem {
  static constexpr int kABytes = kGemmBM * kGemmBK * 2;
  static constexpr int kBBytes = BN * kGemmBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kBarOffset = ST * kStageBytes;
  static constexpr int kTotal = 1024 /*alignment slack*/ + kBarOffset + (2 * ST + 1) * 8 + 16;
  static constexpr uint32_t kTmemCols = BN < 32 ? 32 : BN;
  // partial tile [BN/2 lanes][128 rows] fp32, parked in the drained stage ring
  static_assert(BN / 2 * kGemmBM * 4 <= ST * kStageBytes, "partial tile must fit the ring");
};

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}

__device__ __forceinline__ uint32_t map_to_rank(uint32_t smem_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
  return r;
}

__device__ __forceinline__ float ld_dsmem(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

template <int BN, int ST, int EPI>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                   const __grid_constant__ GemmEpi epi, int Mw, int K, int n_valid, int x_row0,
                   int splits, int* err) {
  using L = GemmSmem<BN, ST>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * ST + 1);
  const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + ST), acc_bar = smem_u32(bars + 2 * ST);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * kGemmBM;          // tile's first output row (store / qkv)
  const int split = blockIdx.y;
  const int n0 = blockIdx.z * BN;               // first activation row of this N tile
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
  // Let the next kernel launch now: it waits (griddepcontrol.wait) for this
  // grid to finish before touching our outputs, but can stage its own
  // weight loads meanwhile.
  pdl_launch_dependents();

  // SwiGLU tiles take rows [64t, 64t+64) of the gate half and the same rows
  // of the up half (two 64-row boxes); other tiles take 128 consecutive rows.
  auto load_w = [&](uint32_t dst, uint32_t bar, int kc) {
    if (EPI == kEpiSwiGLU) {
      const int g0 = blockIdx.x * (kGemmBM / 2);
      tma_load_2d(dst, &tmW, bar, kc, g0);
      tma_load_2d(dst + kGemmBM / 2 * kGemmBK * 2, &tmW, bar, kc, epi.I + g0);
    } else {
      tma_load_2d(dst, &tmW, bar, kc, m0);
    }
  };

  // Weights do not depend on the previous kernel: issue the first ring of
  // weight loads before waiting on it, then the activation loads after.
  if (warp == 0 && lane == 0) {
    const int pre = nkb < ST ? nkb : ST;
    for (int i = 0; i < pre; ++i) {
      const uint32_t fb = full0 + 8 * i;
      mbar_expect_tx(fb, L::kStageBytes);
      load_w(smem_u32(smem + i * L::kStageBytes), fb, (kb0 + i) * kGemmBK);
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
      load_w(smem_u32(st), fb, (kb0 + i) * kGemmBK);
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

  // Park this split's partial tile: red[l][r] = acc[r][2l] + acc[r][2l+1]
  // (lane l's hi and lo activation rows). The ring is drained: every TMA load
  // was consumed by an MMA that completed before acc_bar.
  const bool have = mbar_wait(acc_bar, 0, err, kDevTimeoutAcc);
  tc_fence_after();
  float* red = reinterpret_cast<float*>(smem);
  const int lanes_here = min(BN / 2, n_valid - n0 / 2);   // lanes of this N tile
  {
    const int r = warp * 32 + lane;
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 8) {
      if (c0 / 2 >= lanes_here) break;
      uint32_t v[8];
      tmem_ld_32x32b_x8(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0, v);
      tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float s = (have && nkb > 0) ? __uint_as_float(v[2 * j]) + __uint_as_float(v[2 * j + 1]) : 0.f;
        red[(c0 / 2 + j) * kGemmBM + r] = s;
      }
    }
  }
  tc_fence_before();
  cluster_sync();   // all partial tiles of this m-tile are visible cluster-wide

  // Reduce: this CTA owns units [u0, u1) of the tile's 64 row pairs. A unit is
  // two rows that one epilogue needs together (RoPE pair, gate/up pair, or two
  // adjacent rows).
  const uint32_t my_rank = cluster_rank();
  const int u0 = (int)((long)my_rank * 64 / splits), u1 = (int)((long)(my_rank + 1) * 64 / splits);
  const uint32_t red_base = smem_u32(red);
  for (int item = threadIdx.x; item < (u1 - u0) * lanes_here; item += blockDim.x) {
    const int l = item / (u1 - u0);
    const int u = u0 + item % (u1 - u0);
    int r0, r1;
    if (EPI == kEpiQkvRope) {
      const int half = epi.hd / 2;
      r0 = (u / half) * epi.hd + (u % half);
      r1 = r0 + half;
    } else if (EPI == kEpiSwiGLU) {
      r0 = u;
      r1 = u + kGemmBM / 2;
    } else {
      r0 = 2 * u;
      r1 = 2 * u + 1;
    }
    float v0 = 0.f, v1 = 0.f;
    for (int s = 0; s < splits; ++s) {
      const uint32_t base = map_to_rank(red_base, (uint32_t)s);
      v0 += ld_dsmem(base + (uint32_t)((l * kGemmBM + r0) * 4));
      v1 += ld_dsmem(base + (uint32_t)((l * kGemmBM + r1) * 4));
    }
    const int n = n0 / 2 + l;   // lane index
    if (EPI == kEpiStore) {
      if (m0 + r0 < Mw) epi.out[(long)n * Mw + m0 + r0] = v0;
      if (m0 + r1 < Mw) epi.out[(long)n * Mw + m0 + r1] = v1;
    } else if (EPI == kEpiSwiGLU) {
      const int i = blockIdx.x * (kGemmBM / 2) + u;
      if (i < epi.I) {
        const float a = v0 / (1.f + expf(-v0)) * v1;
        store_pair(epi.x_act, epi.I, n, i, a);
      }
    } else {
      const int hd = epi.hd, half = hd / 2;
      const int mg = m0 + r0;
      const int head = mg / hd, i = mg - head * hd;   // i < half
      const int pos = epi.meta[n * 8 + 1];
      const int slot = epi.meta[n * 8 + 3];
      const int kvd = epi.nkv * hd;
      if (head < epi.nh + epi.nkv) {
        float sn, cs;
        sincosf((float)pos * epi.inv_freq[i], &sn, &cs);
        const float y0 = v0 * cs - v1 * sn, y1 = v1 * cs + v0 * sn;
        if (head < epi.nh) {
          float* qr = epi.q + (long)n * epi.nh * hd + head * hd;
          qr[i] = y0;
          qr[i + half] = y1;
        } else if (slot >= 0 && slot < epi.n_slots) {
          __nv_bfloat16* kr = epi.kpool + (long)slot * kvd + (head - epi.nh) * hd;
          kr[i] = f2bf(y0);
          kr[i + half] = f2bf(y1);
        } else {
          atomicExch(err, kDevBadIndex);
        }
      } else if (slot >= 0 && slot < epi.n_slots) {
        __nv_bfloat16* vr = epi.vpool + (long)slot * kvd + (head - epi.nh - epi.nkv) * hd;
        vr[i] = f2bf(v0);
        vr[i + half] = f2bf(v1);
      }
    }
  }
  cluster_sync();   // no CTA leaves while others still read its partial tile
  if (warp == 2) tmem_dealloc(tmem, L::kTmemCols);
}

}  // namespace ls
