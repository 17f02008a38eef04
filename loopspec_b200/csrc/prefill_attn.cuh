// Prefill attention on tensor cores: many query rows of ONE timeline per CTA.
//
// A prefill role call feeds a chunk of consecutive prompt positions of one
// timeline (one mapping row) as its lanes. The decode kernel (attn_kernel)
// gives every lane its own CTAs, so each lane re-reads the whole K/V prefix;
// here a CTA takes 64 lanes (4 warps x 16 query rows) of one query head and
// streams the timeline's K/V once for all of them, in tiles of 64 positions
// gathered through the mapping row (map[row][t] = KV slot of position t)
// with 16-byte cp.async copies into padded shared-memory rows (double
// buffered), flash-attention style:
//   S = q K^T on mma.sync m16n8k16 bf16 with fp32 accumulation; q is fp32,
//       so it enters as a bf16 (hi, lo) pair and S = q_hi K^T + q_lo K^T
//       (K is stored in bf16, so the products are those of fp32 q);
//   causal mask t <= pos(lane), online softmax per row in fp32 (running max,
//       rescaled sum and accumulator);
//   O += P V with P (fp32) as a (hi, lo) bf16 pair, V fragments by
//       ldmatrix.trans from the [position][dim] tile.
// The reference computes prompt attention with SGLang's extend attention
// over the same paged KV (modeling/ouro.py:37-82 attention, branch KV
// timelines in loopspec/branching/manager.py); the result per row is the
// softmax-weighted mean of V over positions 0..pos, as attn_kernel computes.
// Output: the O GEMM's bf16 (hi, lo) input rows, or fp32 rows.
#pragma once

#include "common.cuh"
#include "kernels.cuh"

namespace ls {

constexpr int kPAttnRows = 64;       // query rows (lanes) per CTA
constexpr int kPAttnKeys = 64;       // positions per K/V tile
constexpr int kPAttnThreads = 128;   // 4 warps x 16 rows

template <int HD>
__host__ __device__ constexpr int pattn_row_bytes() { return HD * 2 + 16; }   // padded: conflict-free fragment loads

template <int HD>
constexpr size_t pattn_smem_bytes() {
  return (size_t)2 * 2 * kPAttnKeys * pattn_row_bytes<HD>();   // 2 buffers x (K, V)
}

__device__ __forceinline__ uint32_t pack_bf16(float lo_elem, float hi_elem) {
  // element 0 (lower column) in the low half, as mma fragments expect
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo_elem, hi_elem);
  return *reinterpret_cast<const uint32_t*>(&v);
}

// (hi, lo) bf16 split of a pair of fp32 values, packed for a fragment register.
__device__ __forceinline__ void split_pair(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  const __nv_bfloat16 h0 = __float2bfloat16_rn(x0), h1 = __float2bfloat16_rn(x1);
  hi = pack_bf16(__bfloat162float(h0), __bfloat162float(h1));
  lo = pack_bf16(x0 - __bfloat162float(h0), x1 - __bfloat162float(h1));
}

__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], const void* p) {
  const uint32_t a = (uint32_t)__cvta_generic_to_shared(p);
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(a));
}


// grid (ceil(n / 64), nh); every lane of the call must share one mapping row.
template <int HD>
__global__ void __launch_bounds__(kPAttnThreads) prefill_attn_kernel(AttnArgs a, int n) {
  static_assert(HD % 16 == 0 && HD <= 128, "head dim");
  constexpr int RB = pattn_row_bytes<HD>();
  constexpr int KS = HD / 16;          // k-steps of S = q K^T
  constexpr int NT = HD / 8;           // n-tiles of O
  constexpr int CH = HD / 8;           // 16-byte chunks per K/V row
  pdl_launch_dependents();
  extern __shared__ __align__(16) unsigned char s_kv[];
  __shared__ int s_slot[2][kPAttnKeys];
  __shared__ int s_pos[kPAttnRows];
  __shared__ int s_tmax;
  const int tile = blockIdx.x, h = blockIdx.y;
  const int G = a.nh / a.nkv, g = h / G;
  const int kd = a.nkv * HD;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gid = lane >> 2, tig = lane & 3;
  const int b0 = tile * kPAttnRows;
  const int row = a.meta.get(kMetaRow, b0);
  if (threadIdx.x == 0) s_tmax = 0;
  __syncthreads();
  if (threadIdx.x < kPAttnRows) {
    const int b = b0 + threadIdx.x;
    int p = -1;
    if (b < n) {
      p = a.meta.get(kMetaPos, b);
      if (p < 0 || p >= a.max_ctx || a.meta.get(kMetaRow, b) != row) {
        atomicExch(a.err, kDevBadIndex);
        p = -1;
      }
    }
    s_pos[threadIdx.x] = p;
    if (p >= 0) atomicMax(&s_tmax, p + 1);
  }
  __syncthreads();
  const int T = s_tmax;
  if (row < 0 || row >= a.rows) {
    if (threadIdx.x == 0) atomicExch(a.err, kDevBadIndex);
    return;
  }
  const int ntiles = (T + kPAttnKeys - 1) / kPAttnKeys;
  const int* map_row = a.map + (long)row * a.max_ctx;

  auto kbuf = [&](int buf) { return s_kv + (size_t)buf * 2 * kPAttnKeys * RB; };
  auto vbuf = [&](int buf) { return s_kv + (size_t)buf * 2 * kPAttnKeys * RB + kPAttnKeys * RB; };
  // slot ids of tile j into s_slot[buf]
  auto load_slots = [&](int j, int buf) {
    if (threadIdx.x < kPAttnKeys) {
      const int t = j * kPAttnKeys + threadIdx.x;
      int sv = -1;
      if (t < T) {
        sv = map_row[t];
        if (sv < 0 || sv >= a.n_slots) {
          atomicExch(a.err, kDevBadIndex);
          sv = -1;
        }
      }
      s_slot[buf][threadIdx.x] = sv;
    }
  };
  auto issue_kv = [&](int buf) {
    unsigned char* kb = kbuf(buf);
    unsigned char* vb = vbuf(buf);
    for (int i = threadIdx.x; i < kPAttnKeys * CH; i += kPAttnThreads) {
      const int r = i / CH, c = i % CH;
      const int sv = s_slot[buf][r];
      const long off = (long)(sv < 0 ? 0 : sv) * kd + g * HD + c * 8;
      cp_async16(kb + r * RB + c * 16, a.kpool + off, sv >= 0);
      cp_async16(vb + r * RB + c * 16, a.vpool + off, sv >= 0);
    }
    cp_async_commit();
  };

  // the slot ids and the mapping are final before this kernel (the mapping
  // update of a prefill call is serialised); q and the chunk's own K/V come
  // from the QKV projection just before
  load_slots(0, 0);
  pdl_wait();
  __syncthreads();
  issue_kv(0);

  // this warp's 16 query rows: q * scale as (hi, lo) A fragments
  const int r0 = warp * 16 + gid, r1 = r0 + 8;
  const int pos0 = s_pos[r0], pos1 = s_pos[r1];
  uint32_t qh[KS][4], ql[KS][4];
  {
    const float* q0 = a.q + (long)(b0 + r0) * a.nh * HD + h * HD;
    const float* q1 = a.q + (long)(b0 + r1) * a.nh * HD + h * HD;
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      const int c = ks * 16 + tig * 2;
      float2 x00 = make_float2(0.f, 0.f), x10 = x00, x01 = x00, x11 = x00;
      if (pos0 >= 0) {
        x00 = *reinterpret_cast<const float2*>(q0 + c);
        x01 = *reinterpret_cast<const float2*>(q0 + c + 8);
      }
      if (pos1 >= 0) {
        x10 = *reinterpret_cast<const float2*>(q1 + c);
        x11 = *reinterpret_cast<const float2*>(q1 + c + 8);
      }
      split_pair(x00.x * a.scale, x00.y * a.scale, qh[ks][0], ql[ks][0]);
      split_pair(x10.x * a.scale, x10.y * a.scale, qh[ks][1], ql[ks][1]);
      split_pair(x01.x * a.scale, x01.y * a.scale, qh[ks][2], ql[ks][2]);
      split_pair(x11.x * a.scale, x11.y * a.scale, qh[ks][3], ql[ks][3]);
    }
  }
  float o[NT][4];
#pragma unroll
  for (int i = 0; i < NT; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

  for (int j = 0; j < ntiles; ++j) {
    const int buf = j & 1;
    if (j + 1 < ntiles) {
      load_slots(j + 1, buf ^ 1);
      __syncthreads();
      issue_kv(buf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const unsigned char* kb = kbuf(buf);
    const unsigned char* vb = vbuf(buf);
    // S = q K^T over the tile's 64 positions (8 n-tiles of 8)
    float s[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
      const unsigned char* kr = kb + (nt * 8 + gid) * RB;
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        const uint32_t kb0 = *reinterpret_cast<const uint32_t*>(kr + (ks * 16 + tig * 2) * 2);
        const uint32_t kb1 = *reinterpret_cast<const uint32_t*>(kr + (ks * 16 + 8 + tig * 2) * 2);
        mma_bf16(s[nt], qh[ks], kb0, kb1);
        mma_bf16(s[nt], ql[ks], kb0, kb1);
      }
    }
    // causal mask and online softmax (rows r0: s[.][0..1], r1: s[.][2..3])
    const int t0 = j * kPAttnKeys;
    float mx0 = m0, mx1 = m1;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int t = t0 + nt * 8 + tig * 2 + e;
        if (t > pos0) s[nt][e] = -INFINITY;
        if (t > pos1) s[nt][2 + e] = -INFINITY;
        mx0 = fmaxf(mx0, s[nt][e]);
        mx1 = fmaxf(mx1, s[nt][2 + e]);
      }
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float c0 = mx0 == -INFINITY ? 1.f : __expf(m0 - mx0);
    const float c1 = mx1 == -INFINITY ? 1.f : __expf(m1 - mx1);
    m0 = mx0;
    m1 = mx1;
    l0 *= c0;
    l1 *= c1;
#pragma unroll
    for (int i = 0; i < NT; ++i) {
      o[i][0] *= c0;
      o[i][1] *= c0;
      o[i][2] *= c1;
      o[i][3] *= c1;
    }
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        s[nt][e] = m0 == -INFINITY ? 0.f : __expf(s[nt][e] - m0);
        s[nt][2 + e] = m1 == -INFINITY ? 0.f : __expf(s[nt][2 + e] - m1);
        l0 += s[nt][e];
        l1 += s[nt][2 + e];
      }
    }
    // O += P V: k-steps of 16 positions; P's A fragment is two S n-tiles
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t ph[4], pl[4];
      split_pair(s[2 * kk][0], s[2 * kk][1], ph[0], pl[0]);
      split_pair(s[2 * kk][2], s[2 * kk][3], ph[1], pl[1]);
      split_pair(s[2 * kk + 1][0], s[2 * kk + 1][1], ph[2], pl[2]);
      split_pair(s[2 * kk + 1][2], s[2 * kk + 1][3], ph[3], pl[3]);
      // lane l addresses row (kk*16 + (l&7) + ((l>>3)&1)*8), columns +((l>>4)*8)
      const int vr = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
      for (int np = 0; np < NT / 2; ++np) {
        uint32_t vf[4];
        ldmatrix_x4_trans(vf, vb + vr * RB + (np * 16 + (lane >> 4) * 8) * 2);
        mma_bf16(o[2 * np], ph, vf[0], vf[1]);
        mma_bf16(o[2 * np], pl, vf[0], vf[1]);
        mma_bf16(o[2 * np + 1], ph, vf[2], vf[3]);
        mma_bf16(o[2 * np + 1], pl, vf[2], vf[3]);
      }
    }
    __syncthreads();   // the buffer is refilled two tiles later
  }
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float inv0 = l0 > 0.f ? 1.f / l0 : 0.f, inv1 = l1 > 0.f ? 1.f / l1 : 0.f;
  const long ld = (long)a.nh * HD;
#pragma unroll
  for (int i = 0; i < NT; ++i) {
    const int col = h * HD + i * 8 + tig * 2;
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      if (pos0 >= 0) {
        if (a.out) a.out[(long)(b0 + r0) * ld + col + e] = o[i][e] * inv0;
        else store_pair(a.x, ld, b0 + r0, col + e, o[i][e] * inv0);
      }
      if (pos1 >= 0) {
        if (a.out) a.out[(long)(b0 + r1) * ld + col + e] = o[i][2 + e] * inv1;
        else store_pair(a.x, ld, b0 + r1, col + e, o[i][2 + e] * inv1);
      }
    }
  }
}

}  // namespace ls
