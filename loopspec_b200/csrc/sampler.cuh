// Fused top-p / top-k / temperature sampling and LoopSpec draft verification.
//
// One CTA (1024 threads) per readout row does, on the device and without a
// host round trip:
//   P = filter(softmax(logits / T)) renormalised (fp32), where top-p keeps
//       every probability >= the largest value v with sum_{p >= v} p >= top_p
//       and top-k every probability >= the k-th largest (ties kept; both ->
//       the larger cutoff), as the reference's sort / cumsum / searchsorted
//       filter (sampling/distributions.py:14-86). The cutoffs are found by
//       bisection over fp32 bit patterns (monotone for non-negative floats)
//       instead of a full sort.
//   q1     draw x ~ P; keep P as the lane's q1 distribution (sampler.py:49-102)
//   q2     r = max(P - Q1, 0), r[x] = 0; draw y ~ r; R = r / sum r; propose y
//          iff sum r > 0 and P[x] < Q1[x] (sampler.py:178-344)
//   final  no q1 token: draw from P; else accept x iff u0 < min(1, P[x]/Q1[x])
//          (sampler.py:428-460); on rejection F = norm(max(P - Q1, 0)), accept
//          the q2 token y iff u1 < min(1, F[y]/R[y]), else draw from
//          norm(max(F - R, 0)) (or F) with u2 (sampling/rejection.py:42-97)
// and writes the decision row (token, proposed, accepted_code, q1_rejected,
// q2_rejected) of policy.py:197-283. Draws invert a CDF in chunks of 2048
// tokens like the reference. Uniforms: words of Philox4x32-10 with counter
// (cycle, readout row of the request, 0, 0) and the request's seed as key,
// u = (w >> 8) * 2^-24 (cycle, row and seed come with the row's metadata).
#pragma once

#include "common.cuh"
#include "kernels.cuh"

namespace ls {

constexpr int kSampleThreads = 1024;
constexpr int kSampleChunk = 2048;
constexpr int kSampleMaxChunks = 64;        // vocab <= 131072
constexpr int kSampleSmemVocab = 51200;     // P kept in shared memory up to this vocab

struct SampleParams {
  float temperature;
  float top_p;
  int top_k;
  int pad;
  unsigned long long seed;
};

struct SampleArgs {
  Meta meta;                    // readout rows: kind, first, second, state slot, cycle
  int meta_row0;                // metadata record of row 0 (head lanes may start later)
  const float* logits;          // [rows][V]
  int V;
  const SampleParams* params;   // device copy (graphs read it at run time)
  float* q1_bank;               // [bank_rows][V] lane q1 distributions, by state slot
  float* r_bank;                // [bank_rows][V] lane q2 residual distributions
  int bank_rows;
  float* work;                  // [rows][2][V] scratch (P when it does not fit smem, and W)
  long long* decisions;         // [rows][5]
  int* err;
};

__device__ __forceinline__ uint4 philox_words(unsigned long long seed, uint32_t c0, uint32_t c1) {
  return philox4x32_10(make_uint4(c0, c1, 0u, 0u), (uint32_t)seed, (uint32_t)(seed >> 32));
}

// Deterministic block reductions over 1024 threads (fixed tree).
__device__ __forceinline__ float sblock_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.f;
  return warp_sum(t);
}

__device__ __forceinline__ float sblock_max(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = lane < (int)(blockDim.x >> 5) ? red[lane] : -INFINITY;
  return warp_max(t);
}

// Row loops visit E consecutive elements per step (E = 4 when V % 4 == 0: one
// 16-byte load or store per step, else 1): thread tid takes steps tid,
// tid + blockDim.x, ... and, within a step, elements in index order. A row's
// sums are therefore a fixed function of the row.
template <int E>
struct Vf {
  float v[E];
};

template <int E>
__device__ __forceinline__ Vf<E> ldv(const float* p, int j) {
  Vf<E> x;
  if constexpr (E == 4) {
    const float4 q = *reinterpret_cast<const float4*>(p + 4 * j);
    x.v[0] = q.x;
    x.v[1] = q.y;
    x.v[2] = q.z;
    x.v[3] = q.w;
  } else {
    x.v[0] = p[j];
  }
  return x;
}

template <int E>
__device__ __forceinline__ void stv(float* p, int j, const Vf<E>& x) {
  if constexpr (E == 4) *reinterpret_cast<float4*>(p + 4 * j) = make_float4(x.v[0], x.v[1], x.v[2], x.v[3]);
  else p[j] = x.v[0];
}

// Largest value v (an element of p) with F(v) >= target, F(v) = sum or count
// of the elements >= v, found by bisection over the bit patterns in [0, max].
template <bool COUNT, int E>
__device__ float bisect_cutoff(const float* p, int V, float target, float pmax, float* red) {
  uint32_t lo = 0u, hi = __float_as_uint(pmax) + 1u;   // F(lo) >= target > F(hi)
  while (hi - lo > 1u) {
    const uint32_t mid = lo + (hi - lo) / 2u;
    const float v = __uint_as_float(mid);
    float acc = 0.f;
#pragma unroll 4
    for (int j = threadIdx.x; j < V / E; j += blockDim.x) {
      const Vf<E> x = ldv<E>(p, j);
#pragma unroll
      for (int i = 0; i < E; ++i)
        if (x.v[i] >= v) acc += COUNT ? 1.f : x.v[i];
    }
    const float tot = sblock_sum(acc, red);
    if (tot >= target) lo = mid;
    else hi = mid;
  }
  return __uint_as_float(lo);
}

// Inverse-CDF draw from non-negative weights w (need not be normalised).
// target = u * total; first 2048-chunk whose inclusive CDF exceeds target, then
// the first token of it whose inclusive CDF exceeds target - preceding mass.
//
// A chunk is walked as 64 rows of 32 consecutive tokens, one token per lane
// (consecutive lanes read consecutive words: no shared-memory bank conflicts),
// with a warp prefix scan per row and the row totals added in row order. The
// chunk totals and the in-chunk search use this same order, so the chunk the
// totals pick always contains the crossing.
__device__ __forceinline__ float warp_incl_scan(float x) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  return x;
}

__device__ __forceinline__ float chunk_total(const float* w, int c, int V) {
  const int lane = threadIdx.x & 31;
  float tot = 0.f;
  for (int i0 = 0; i0 < kSampleChunk / 32; i0 += 8) {
    float x[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int t = c * kSampleChunk + (i0 + j) * 32 + lane;
      x[j] = t < V ? w[t] : 0.f;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) tot += __shfl_sync(0xffffffffu, warp_incl_scan(x[j]), 31);
  }
  return tot;
}

__device__ int block_pick(const float* w, int V, float u, float* s_chunk, float* red, int* s_idx) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int nch = (V + kSampleChunk - 1) / kSampleChunk;
  for (int c = warp; c < nch; c += nw) {          // one warp per chunk
    const float a = chunk_total(w, c, V);
    if (lane == 0) s_chunk[c] = a;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float total = 0.f;
    for (int c = 0; c < nch; ++c) total += s_chunk[c];
    const float target = u * total;
    float cdf = 0.f, pre = 0.f;
    int ch = -1;
    for (int c = 0; c < nch; ++c) {
      if (cdf + s_chunk[c] > target) {
        ch = c;
        pre = cdf;
        break;
      }
      cdf += s_chunk[c];
    }
    if (ch < 0) {
      ch = 0;
      pre = 0.f;
    }
    s_idx[0] = ch;
    red[0] = target - pre;
  }
  __syncthreads();
  const int ch = s_idx[0];
  const float rem = red[0];
  __syncthreads();
  if (warp == 0) {
    int found = -1;                                  // nothing exceeds: first token of the chunk
    float pre = 0.f;
    for (int i0 = 0; i0 < kSampleChunk / 32 && found < 0; i0 += 8) {
      float x[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int t = ch * kSampleChunk + (i0 + j) * 32 + lane;
        x[j] = t < V ? w[t] : 0.f;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (found < 0) {                             // warp-uniform
          const float incl = warp_incl_scan(x[j]);
          const unsigned hit = __ballot_sync(0xffffffffu, pre + incl > rem);
          if (hit) found = ch * kSampleChunk + (i0 + j) * 32 + (__ffs(hit) - 1);
          else pre += __shfl_sync(0xffffffffu, incl, 31);
        }
      }
    }
    if (lane == 0) s_idx[1] = found >= 0 ? found : ch * kSampleChunk;
  }
  __syncthreads();
  const int r = s_idx[1];
  __syncthreads();
  return r;
}

template <bool SMEM_P, int E>
__global__ void __launch_bounds__(kSampleThreads) sample_kernel(SampleArgs a) {
  pdl_launch_dependents();
  pdl_wait();
  extern __shared__ __align__(16) float s_p[];
  __shared__ float red[32];
  __shared__ float s_chunk[kSampleMaxChunks];
  __shared__ int s_idx[2];
  const int row = blockIdx.x;
  const int V = a.V;
  const SampleParams prm = *a.params;
  const int kind = a.meta.get(kMetaKind, a.meta_row0 + row);
  const int first = a.meta.get(kMetaFirst, a.meta_row0 + row);
  const int second = a.meta.get(kMetaSecond, a.meta_row0 + row);
  const int slot = a.meta.get(kMetaStateIn, a.meta_row0 + row);
  const uint32_t cycle = (uint32_t)a.meta.get(kMetaCycle, a.meta_row0 + row);
  float* P = SMEM_P ? s_p : a.work + (long)row * 2 * V;
  float* W = a.work + (long)row * 2 * V + V;
  const float* lg = a.logits + (long)row * V;
  const bool need_bank = kind == 0 || kind == 1 || first >= 0;
  if (need_bank && (slot < 0 || slot >= a.bank_rows)) {
    if (threadIdx.x == 0) atomicExch(a.err, kDevBadIndex);
    return;
  }
  if ((first >= V) || (second >= V) || ((kind == 1) && first < 0)) {
    if (threadIdx.x == 0) atomicExch(a.err, kDevBadIndex);
    return;
  }

  // softmax(logits / T) in fp32
  const int NV = V / E, tid = threadIdx.x, nt = blockDim.x;
  const float invT = 1.f / prm.temperature;
  float m = -INFINITY;
#pragma unroll 4
  for (int j = tid; j < NV; j += nt) {
    const Vf<E> x = ldv<E>(lg, j);
#pragma unroll
    for (int i = 0; i < E; ++i) m = fmaxf(m, x.v[i] * invT);
  }
  m = sblock_max(m, red);
  float s = 0.f;
#pragma unroll 4
  for (int j = tid; j < NV; j += nt) {
    Vf<E> x = ldv<E>(lg, j);
#pragma unroll
    for (int i = 0; i < E; ++i) {
      x.v[i] = expf(x.v[i] * invT - m);
      s += x.v[i];
    }
    stv<E>(P, j, x);
  }
  s = sblock_sum(s, red);
  float pmax = 0.f;
#pragma unroll 4
  for (int j = tid; j < NV; j += nt) {
    Vf<E> x = ldv<E>(P, j);
#pragma unroll
    for (int i = 0; i < E; ++i) {
      x.v[i] = x.v[i] / s;
      pmax = fmaxf(pmax, x.v[i]);
    }
    stv<E>(P, j, x);
  }
  pmax = sblock_max(pmax, red);
  // top-k / top-p cutoffs, then renormalise over the kept support
  const int k = prm.top_k >= V ? 0 : prm.top_k;
  if (k > 0 || prm.top_p < 1.f) {
    float cut = 0.f;
    if (prm.top_p < 1.f) cut = bisect_cutoff<false, E>(P, V, prm.top_p, pmax, red);
    if (k > 0) cut = fmaxf(cut, bisect_cutoff<true, E>(P, V, (float)k, pmax, red));
    float kept = 0.f;
#pragma unroll 4
    for (int j = tid; j < NV; j += nt) {
      Vf<E> x = ldv<E>(P, j);
#pragma unroll
      for (int i = 0; i < E; ++i) {
        x.v[i] = x.v[i] >= cut ? x.v[i] : 0.f;
        kept += x.v[i];
      }
      stv<E>(P, j, x);
    }
    kept = sblock_sum(kept, red);
#pragma unroll 4
    for (int j = tid; j < NV; j += nt) {
      Vf<E> x = ldv<E>(P, j);
#pragma unroll
      for (int i = 0; i < E; ++i) x.v[i] = x.v[i] / kept;
      stv<E>(P, j, x);
    }
  }
  __syncthreads();

  // the request's stream: its seed, cycle counter and readout row
  const unsigned long long seed =
      (unsigned long long)(uint32_t)a.meta.get(kMetaSeedLo, a.meta_row0 + row) |
      ((unsigned long long)(uint32_t)a.meta.get(kMetaSeedHi, a.meta_row0 + row) << 32);
  const uint32_t draw_row = (uint32_t)a.meta.get(kMetaDrawRow, a.meta_row0 + row);
  const uint4 w4 = philox_words(seed, cycle, draw_row);
  const float u0 = (float)(w4.x >> 8) * (1.f / 16777216.f);
  const float u1 = (float)(w4.y >> 8) * (1.f / 16777216.f);
  const float u2 = (float)(w4.z >> 8) * (1.f / 16777216.f);
  long long d[5] = {0, 0, 0, 0, 0};

  if (kind == 0) {                                     // q1: draw and keep P
    float* q1 = a.q1_bank + (long)slot * V;
#pragma unroll 4
    for (int j = tid; j < NV; j += nt) stv<E>(q1, j, ldv<E>(P, j));
    d[0] = block_pick(P, V, u0, s_chunk, red, s_idx);
    d[1] = 1;
  } else if (kind == 1) {                              // q2: conditional residual
    const float* q1 = a.q1_bank + (long)slot * V;
    float mass = 0.f;
#pragma unroll 4
    for (int j = tid; j < NV; j += nt) {
      const Vf<E> p = ldv<E>(P, j), q = ldv<E>(q1, j);
      Vf<E> r;
#pragma unroll
      for (int i = 0; i < E; ++i) {
        r.v[i] = j * E + i == first ? 0.f : fmaxf(p.v[i] - q.v[i], 0.f);
        mass += r.v[i];
      }
      stv<E>(W, j, r);
    }
    mass = sblock_sum(mass, red);
    const int y = block_pick(W, V, u0, s_chunk, red, s_idx);
    float* R = a.r_bank + (long)slot * V;
#pragma unroll 4
    for (int j = tid; j < NV; j += nt) {
      Vf<E> r = ldv<E>(W, j);
#pragma unroll
      for (int i = 0; i < E; ++i) r.v[i] = mass > 0.f ? r.v[i] / mass : 0.f;
      stv<E>(R, j, r);
    }
    const int action = mass > 0.f && P[first] < q1[first];
    d[0] = action ? y : first;
    d[1] = action;
    d[2] = action;
  } else if (first < 0) {                              // final without a proposal
    d[0] = block_pick(P, V, u0, s_chunk, red, s_idx);
  } else {                                             // final verification
    const float* q1 = a.q1_bank + (long)slot * V;
    const float acc = fminf(1.f, P[first] / q1[first]);
    if (u0 < acc) {
      d[0] = first;
      d[2] = 1;
    } else {
      float mF = 0.f, mP = 0.f;
#pragma unroll 4
      for (int j = tid; j < NV; j += nt) {
        const Vf<E> p = ldv<E>(P, j), q = ldv<E>(q1, j);
        Vf<E> f;
#pragma unroll
        for (int i = 0; i < E; ++i) {
          f.v[i] = fmaxf(p.v[i] - q.v[i], 0.f);
          mF += f.v[i];
          mP += p.v[i];
        }
        stv<E>(W, j, f);
      }
      mF = sblock_sum(mF, red);
      mP = sblock_sum(mP, red);
#pragma unroll 4
      for (int j = tid; j < NV; j += nt) {
        Vf<E> f = ldv<E>(W, j);
        const Vf<E> p = ldv<E>(P, j);
#pragma unroll
        for (int i = 0; i < E; ++i) f.v[i] = mF > 0.f ? f.v[i] / mF : p.v[i] / (mP > 0.f ? mP : 1.f);
        stv<E>(W, j, f);
      }
      __syncthreads();
      bool acc2 = false;
      if (second >= 0) {
        const float* R = a.r_bank + (long)slot * V;
        acc2 = u1 < fminf(1.f, W[second] / R[second]);
        float mG = 0.f;
#pragma unroll 4
        for (int j = tid; j < NV; j += nt) {
          const Vf<E> f = ldv<E>(W, j), r = ldv<E>(R, j);
#pragma unroll
          for (int i = 0; i < E; ++i) mG += fmaxf(f.v[i] - r.v[i], 0.f);
        }
        mG = sblock_sum(mG, red);
        if (mG > 0.f) {
#pragma unroll 4
          for (int j = tid; j < NV; j += nt) {
            Vf<E> f = ldv<E>(W, j);
            const Vf<E> r = ldv<E>(R, j);
#pragma unroll
            for (int i = 0; i < E; ++i) f.v[i] = fmaxf(f.v[i] - r.v[i], 0.f) / mG;
            stv<E>(W, j, f);
          }
        }
        __syncthreads();
      }
      const int smp = block_pick(W, V, u2, s_chunk, red, s_idx);
      d[0] = acc2 ? second : smp;
      d[2] = acc2 ? 2 : 0;
      d[3] = 1;
      d[4] = second >= 0 && !acc2;
    }
  }
  if (threadIdx.x == 0) {
#pragma unroll
    for (int i = 0; i < 5; ++i) a.decisions[(long)row * 5 + i] = d[i];
  }
}

}  // namespace ls
