// Weight-streaming GEMM on 5th-generation tensor cores (sm_100a) with a
// last-split split-K reduction and fused epilogues.
//
//   y[n][m] = sum_k W[m][k] * x[n][k]
//
// W is a bf16 weight [Mw, K] (row-major, K contiguous); x is the lane
// activation, stored as a bf16 (hi, lo) row pair per lane in X [2*Ncap, K]
// starting at row x_row0. Weight rows fill the 128-row M side of
// tcgen05.mma and activation rows sit on N (16..256), so a handful of decode
// lanes still uses the full tensor-core M width.
//
// Grid (m_tiles, splits, n_tiles): the `splits` CTAs of one m-tile each
// stream a fixed K range (boundaries depend only on K and splits, never on the
// batch). TMA streams 128x64 weight boxes and BNx64 activation boxes into an
// ST-deep shared-memory ring (128-byte swizzle); one thread issues the MMAs
// into a TMEM accumulator; four warps read it back and add each lane's hi/lo
// columns. The last split of a tile to finish (atomic ticket) sums the splits'
// partial tiles in split order and applies the epilogue. (Clusters with a
// DSMEM reduction were measured slower: only 15 eight-CTA clusters fit on the
// GPU at once, which split the GEMMs into two waves.)
//   kEpiStore   y -> fp32 out[n][m]
//   kEpiStoreArgmax  (lm_head, one split) kEpiStore, and each lane's
//               (max, lowest index of the max) over the tile's rows; the last
//               CTA of the grid to finish (acquire-release ticket) reduces the
//               tiles' pairs into each lane's greedy token, so no separate
//               pass re-reads the [lanes][vocab] logits (torch.argmax
//               semantics, sglang_recurrent/loopspec/decisions.py:116)
//   kEpiQkvRope q/k rows get neox RoPE at the lane's position; k and v go to
//               the layer's KV pool at the lane's slot (bf16), q to fp32
//   kEpiSwiGLU  the tile holds 64 gate rows and their 64 up rows (two TMA
//               boxes); writes silu(g) * u as the next GEMM's (hi, lo) input
//   kEpiSplitStore  every split writes its partial tile to its own plane,
//               out[split * split_stride + n * Mw + m], and exits: no ticket,
//               no re-read. The consumer (a per-lane row kernel) adds the
//               planes in split order while it loads the row.
// A lane's result therefore never depends on the batch it runs in.
#pragma once

#include "common.cuh"

namespace ls {

constexpr int kGemmBM = 128;
constexpr int kGemmBK = 64;   // 64 bf16 = 128 bytes = one swizzle row
constexpr int kGemmThreads = 128;
constexpr int kMaxSplits = 32; // K splits per 128-row tile

enum GemmEpiKind : int { kEpiStore = 0, kEpiQkvRope = 1, kEpiSwiGLU = 2, kEpiSplitStore = 3,
                         kEpiStoreArgmax = 4, kEpiClusterStore = 5 };

// kEpiClusterStore: the K splits of one output tile form a thread-block
// cluster (1, splits, 1); each parks its partial tile in shared memory, and
// after a cluster barrier split r adds every split's values for its 1/splits
// of the tile, in split order, through distributed shared memory and writes
// the one summed plane. The consumer reads one plane instead of `splits`.
constexpr int kMaxClusterSplits = 16;   // non-portable cluster size

__device__ __forceinline__ void gemm_cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ float gemm_ld_cluster(const float* p, uint32_t rank) {
  const uint32_t a = (uint32_t)__cvta_generic_to_shared(p);
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(rank));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(r) : "memory");
  return v;
}

struct GemmEpi {
  float* out;                 // store: out[n * Mw + m]
  const int* meta;            // qkv: lane metadata (int32 [cap][kMetaFields])
  const float* inv_freq;      // qkv: [hd/2]
  float* q;                   // qkv: [cap][nh*hd]
  __nv_bfloat16* kpool;       // qkv: this layer's [slots][nkv*hd]
  __nv_bfloat16* vpool;
  int hd, nh, nkv, n_slots;
  __nv_bfloat16* x_act;       // swiglu: (hi, lo) rows [2*cap][I]
  int I;
  float* part_ws;             // split partial tiles [tiles][splits][BN/2][128] (splits > 1)
  int* tile_tickets;          // [tiles], zero between launches
  float* amax_val;            // argmax: per-lane tile maxima [lanes][m_tiles]
  int* amax_idx;              // ... and their row indices
  int* amax_ticket;           // ... one counter, zero between launches
  long long* amax_out;        // ... each lane's token [lanes]
  long split_stride;          // split store: floats between split planes of out
  const int* active;          // device-resident loop: number of live lanes of the call (a prefix
                              // of the n_valid lanes), read at run time; null: all n_valid
  // split store into a tensor-parallel exchange region: the last CTA to
  // finish advances this rank's epoch and raises its flag (null: no publish)
  int* pub_epoch;
  int* pub_flag;
  int* pub_ticket;            // zero between launches
};

// SUB 64-wide sub-tiles per ring stage along K: the MMA thread's per-stage
// cost (barrier wait, commit) is paid once per SUB k-blocks.
template <int BN, int ST, int SUB = 1>
struct GemmSmem {
  static constexpr int kSubA = kGemmBM * kGemmBK * 2;
  static constexpr int kSubB = BN * kGemmBK * 2;
  static constexpr int kABytes = kSubA * SUB;
  static constexpr int kBBytes = kSubB * SUB;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kBarOffset = ST * kStageBytes;
  static constexpr int kTotal = 1024 /*alignment slack*/ + kBarOffset + (2 * ST + 1) * 8 + 16;
  static constexpr uint32_t kTmemCols = BN < 32 ? 32 : BN;
  // partial tile [BN/2 lanes][128 rows] fp32, parked in the drained stage ring
  static_assert(BN / 2 * kGemmBM * 4 <= ST * kStageBytes, "partial tile must fit the ring");
};

template <int BN, int ST, int EPI, int SUB = 1>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                   const __grid_constant__ GemmEpi epi, int Mw, int K, int n_valid, int x_row0,
                   int splits, int* err) {
  using L = GemmSmem<BN, ST, SUB>;
  constexpr int UK = kGemmBK * SUB;   // k elements per ring stage
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
  const int KB = (K + UK - 1) / UK;   // k-units (split boundaries in units)
  const int kb0 = (int)((long)split * KB / splits);
  const int kb1 = (int)((long)(split + 1) * KB / splits);
  const int nkb = kb1 - kb0;
  // live lanes: the epilogue skips the inactive tail of a fixed-width call
  // (the count was written before this graph started; read it early)
  const int n_live = epi.active ? max(0, min(n_valid, __ldcg(epi.active))) : n_valid;

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
  auto load_w = [&](uint32_t dst0, uint32_t bar, int kc0) {
#pragma unroll
    for (int u = 0; u < SUB; ++u) {   // past K: the box reads the zero fill
      const uint32_t dst = dst0 + u * L::kSubA;
      const int kc = kc0 + u * kGemmBK;
      if (EPI == kEpiSwiGLU) {
        const int g0 = blockIdx.x * (kGemmBM / 2);
        tma_load_2d(dst, &tmW, bar, kc, g0);
        tma_load_2d(dst + kGemmBM / 2 * kGemmBK * 2, &tmW, bar, kc, epi.I + g0);
      } else {
        tma_load_2d(dst, &tmW, bar, kc, m0);
      }
    }
  };
  auto load_x = [&](uint32_t dst0, uint32_t bar, int kc0) {
#pragma unroll
    for (int u = 0; u < SUB; ++u)
      tma_load_2d(dst0 + u * L::kSubB, &tmX, bar, kc0 + u * kGemmBK, x_row0 + n0);
  };

  // Weights do not depend on the previous kernel: issue the first ring of
  // weight loads before waiting on it, then the activation loads after.
  if (warp == 0 && lane == 0) {
    const int pre = nkb < ST ? nkb : ST;
    for (int i = 0; i < pre; ++i) {
      const uint32_t fb = full0 + 8 * i;
      mbar_expect_tx(fb, L::kStageBytes);
      load_w(smem_u32(smem + i * L::kStageBytes), fb, (kb0 + i) * UK);
    }
    pdl_wait();
    for (int i = 0; i < pre; ++i)
      load_x(smem_u32(smem + i * L::kStageBytes + L::kABytes), full0 + 8 * i, (kb0 + i) * UK);
    for (int i = pre; i < nkb; ++i) {
      const int s = i % ST;
      const uint32_t ph = (uint32_t)((i / ST) & 1);
      if (!mbar_wait(empty0 + 8 * s, ph ^ 1u, err, kDevTimeoutEmpty)) break;
      const uint32_t fb = full0 + 8 * s;
      mbar_expect_tx(fb, L::kStageBytes);
      uint8_t* st = smem + s * L::kStageBytes;
      load_w(smem_u32(st), fb, (kb0 + i) * UK);
      load_x(smem_u32(st + L::kABytes), fb, (kb0 + i) * UK);
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
      for (int u = 0; u < SUB; ++u)
#pragma unroll
        for (int k = 0; k < kGemmBK / 16; ++k)
          tc_mma_bf16(tmem, umma_desc_sw128(a + u * L::kSubA + 32 * k), umma_desc_sw128(b + u * L::kSubB + 32 * k),
                      idesc, (i | u | k) != 0);
      tc_commit(empty0 + 8 * s);
    }
    tc_commit(acc_bar);
  }
  __syncthreads();

  // Park this split's partial tile in shared memory: red[l][r] = acc[r][2l] +
  // acc[r][2l+1] (lane l's hi and lo activation rows). With K splits, each
  // split also publishes the tile to global scratch and takes a ticket; the
  // last split of the tile to finish sums all splits in split order (so the
  // result does not depend on which split finished last) and runs the
  // epilogue while the others exit. The ring is drained: every TMA load was
  // consumed by an MMA that completed before acc_bar.
  const bool have = mbar_wait(acc_bar, 0, err, kDevTimeoutAcc);
  tc_fence_after();
  float* red = reinterpret_cast<float*>(smem);
  const int lanes_here = min(BN / 2, n_live - n0 / 2);   // lanes of this N tile
  const long tile_id = (long)blockIdx.z * gridDim.x + blockIdx.x;
  const long split_floats = (long)(BN / 2) * kGemmBM;
  float* tile_part = epi.part_ws + tile_id * splits * split_floats;
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
        if (EPI == kEpiSplitStore) {
          if (m0 + r < Mw && c0 / 2 + j < lanes_here)
            epi.out[split * epi.split_stride + (long)(n0 / 2 + c0 / 2 + j) * Mw + m0 + r] = s;
          continue;
        }
        red[(c0 / 2 + j) * kGemmBM + r] = s;
        if (EPI != kEpiClusterStore && splits > 1)
          tile_part[split * split_floats + (c0 / 2 + j) * kGemmBM + r] = s;
      }
    }
  }
  tc_fence_before();
  __shared__ int s_last;
  __syncthreads();
  if (warp == 2) tmem_dealloc(tmem, L::kTmemCols);
  if (EPI == kEpiClusterStore) {
    // every CTA of the cluster reaches both barriers (lanes_here is the same
    // for all splits of a tile)
    gemm_cluster_sync();   // every split's partial tile is parked
    const int E = max(0, lanes_here) * kGemmBM;
    const int e0 = (int)((long)split * E / splits), e1 = (int)((long)(split + 1) * E / splits);
    for (int e = e0 + (int)threadIdx.x; e < e1; e += blockDim.x) {
      float v[kMaxClusterSplits];
#pragma unroll
      for (int s = 0; s < kMaxClusterSplits; ++s) v[s] = s < splits ? gemm_ld_cluster(red + e, (uint32_t)s) : 0.f;
      float t = 0.f;
#pragma unroll
      for (int s = 0; s < kMaxClusterSplits; ++s)
        if (s < splits) t += v[s];
      const int l = e / kGemmBM, rr = e - l * kGemmBM;
      if (m0 + rr < Mw) epi.out[(long)(n0 / 2 + l) * Mw + m0 + rr] = t;
    }
    gemm_cluster_sync();   // no CTA leaves while another may still read its tile
    return;
  }
  if (EPI == kEpiSplitStore) {
    if (epi.pub_flag && threadIdx.x == 0) {
      // the barrier above ordered the CTA's plane stores before this thread's
      // system-scope fence; the last CTA's fence after its ticket orders every
      // CTA's stores before the flag the peers acquire
      __threadfence_system();
      const int total = gridDim.x * gridDim.y * gridDim.z;
      if (atomicAdd(epi.pub_ticket, 1) == total - 1) {
        __threadfence_system();
        *epi.pub_ticket = 0;   // ready for the next launch
        const int ep = atomicAdd(epi.pub_epoch, 1) + 1;
        asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(epi.pub_flag), "r"(ep) : "memory");
      }
    }
    return;
  }
  if (splits > 1) {
    if (threadIdx.x == 0) {
      int* tk = epi.tile_tickets + tile_id;
      const int t = ticket_take(tk);
      s_last = t == splits - 1;
      if (s_last) *tk = 0;   // every split has arrived: ready for the next launch
    }
    __syncthreads();
    if (!s_last) return;
  }

  // Epilogue over the tile's 64 row pairs. A unit is two rows that one
  // epilogue needs together (RoPE pair, gate/up pair, or two adjacent rows).
  for (int item = threadIdx.x; item < 64 * lanes_here; item += blockDim.x) {
    const int l = item / 64;
    const int u = item % 64;
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
    if (splits == 1) {
      v0 = red[l * kGemmBM + r0];
      v1 = red[l * kGemmBM + r1];
    } else {
      // issue every split's loads first, then add them in split order
      float a0[kMaxSplits], a1[kMaxSplits];
#pragma unroll
      for (int s = 0; s < kMaxSplits; ++s) {
        if (s < splits) {
          const float* ps = tile_part + s * split_floats + l * kGemmBM;
          a0[s] = s == split ? red[l * kGemmBM + r0] : __ldcg(ps + r0);
          a1[s] = s == split ? red[l * kGemmBM + r1] : __ldcg(ps + r1);
        }
      }
#pragma unroll
      for (int s = 0; s < kMaxSplits; ++s) {
        if (s < splits) {
          v0 += a0[s];
          v1 += a1[s];
        }
      }
    }
    const int n = n0 / 2 + l;   // lane index
    if (EPI == kEpiStore || EPI == kEpiStoreArgmax) {
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
      const int pos = epi.meta[n * kMetaFields + kMetaPos];
      const int slot = epi.meta[n * kMetaFields + kMetaSlot];
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
  if (EPI == kEpiStoreArgmax) {
    // each lane's best row of this tile: warp w takes lanes w, w + 4, ...;
    // its 32 threads scan rows r, r + 32, r + 64, r + 96 and shuffle-reduce
    // (larger value first, then the lower row on ties)
    const int tiles = gridDim.x;
    for (int l = warp; l < lanes_here; l += kGemmThreads / 32) {
      float best = -INFINITY;
      int bi = 0x7fffffff;
      for (int r = lane; r < kGemmBM; r += 32) {
        if (m0 + r >= Mw) break;
        const float x = red[l * kGemmBM + r];
        if (x > best || (x == best && m0 + r < bi)) {
          best = x;
          bi = m0 + r;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ob > best || (ob == best && oi < bi)) {
          best = ob;
          bi = oi;
        }
      }
      if (lane == 0) {
        const long at = (long)(n0 / 2 + l) * tiles + blockIdx.x;
        epi.amax_val[at] = best;
        epi.amax_idx[at] = bi;
      }
    }
    __shared__ int s_final;
    __syncthreads();
    if (threadIdx.x == 0) {
      const int total = gridDim.x * gridDim.z;
      const int t = ticket_take(epi.amax_ticket);
      s_final = t == total - 1;
      if (s_final) *epi.amax_ticket = 0;   // every CTA has arrived: ready for the next launch
    }
    __syncthreads();
    if (!s_final) return;
    // last CTA: reduce every lane over all tiles (L2 loads: other CTAs wrote them)
    for (int l = warp; l < n_live; l += kGemmThreads / 32) {
      float best = -INFINITY;
      int bi = 0x7fffffff;
      for (int t = lane; t < tiles; t += 32) {
        const float x = __ldcg(epi.amax_val + (long)l * tiles + t);
        const int xi = __ldcg(epi.amax_idx + (long)l * tiles + t);
        if (x > best || (x == best && xi < bi)) {
          best = x;
          bi = xi;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ob > best || (ob == best && oi < bi)) {
          best = ob;
          bi = oi;
        }
      }
      if (lane == 0) epi.amax_out[l] = bi == 0x7fffffff ? 0 : bi;
    }
  }
}

}  // namespace ls
