// Fused top-p / top-k / temperature sampling and LoopSpec draft verification.
//
// One thread-block cluster of C CTAs (C = min(8, chunks)) per readout row;
// CTA r owns the vocabulary chunks [r*nch/C, (r+1)*nch/C) of 2048 tokens and
// keeps its slice of the row in shared memory. Row-wide sums and maxima are
// block reductions whose per-CTA results every CTA reads from the others'
// shared memory after a cluster barrier, always in rank order, so every CTA
// holds the same value and a row's result is a fixed function of the row.
// On the device and without a host round trip the cluster does:
//   P = filter(softmax(logits / T)) renormalised (fp32), where top-p keeps
//       every probability >= the largest value v with sum_{p >= v} p >= top_p
//       and top-k every probability >= the k-th largest (ties kept; both ->
//       the larger cutoff), as the reference's sort / cumsum / searchsorted
//       filter (sampling/distributions.py:14-86). Each cutoff is found over
//       the fp32 bit patterns (monotone for non-negative floats) in 6 passes
//       of a 33-bin histogram (32 bins of width 2^s over [lo, lo + 2^(s+5))
//       and one above), each pass narrowing the bracket to one bin, instead of
//       a full sort; the last pass also gives the kept mass.
//   q1     draw x ~ P; keep P as the lane's q1 distribution (sampler.py:49-102)
//   q2     r = max(P - Q1, 0), r[x] = 0; draw y ~ r; R = r / sum r; propose y
//          iff sum r > 0 and P[x] < Q1[x] (sampler.py:178-344)
//   final  no q1 token: draw from P; else accept x iff u0 < min(1, P[x]/Q1[x])
//          (sampler.py:428-460); on rejection F = norm(max(P - Q1, 0)), accept
//          the q2 token y iff u1 < min(1, F[y]/R[y]), else draw from
//          norm(max(F - R, 0)) (or F) with u2 (sampling/rejection.py:42-97)
// and writes the decision row (token, proposed, accepted_code, q1_rejected,
// q2_rejected) of policy.py:197-283. A row whose request decodes greedily
// (top_k == 1) in a batch with sampled requests takes the argmax of its
// logits (lowest index on ties, as the greedy path) as the row's token.
// Single probabilities (P[x], F[y]) are recomputed by every CTA from the
// logits with the slice loops' operations, so every CTA takes the same
// branch. Draws invert a CDF in chunks of 2048
// tokens like the reference. Uniforms: words of Philox4x32-10 with counter
// (cycle, readout row of the request, 0, 0) and the request's seed as key,
// u = (w >> 8) * 2^-24 (cycle, row and seed come with the row's metadata).
#pragma once

#include "common.cuh"
#include "kernels.cuh"

namespace ls {

constexpr int kSampleThreads = 512;
constexpr int kSampleChunk = 2048;
constexpr int kSampleMaxChunks = 64;        // vocab <= 131072
constexpr int kSampleCtas = 8;              // CTAs per row (one portable cluster) at most
constexpr int kSampleBins = 32;             // cutoff search: bins per pass (plus one above)
constexpr int kSampleBinShift = 5;          // log2(kSampleBins)

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
  const SampleParams* params;   // per-request slots, device copies (graphs read them at run time)
  int n_params;
  float* q1_bank;               // [bank_rows][V] lane q1 distributions, by state slot
  float* r_bank;                // [bank_rows][V] lane q2 residual distributions
  int bank_rows;
  long long* decisions;         // [rows][5]
  int* err;
};

// Vocabulary split of a row over its cluster (host and device agree).
__host__ __device__ inline int sample_chunks(int V) { return (V + kSampleChunk - 1) / kSampleChunk; }
__host__ __device__ inline int sample_ctas(int V) {
  const int n = sample_chunks(V);
  return n < kSampleCtas ? n : kSampleCtas;
}
__host__ __device__ inline int sample_chunk0(int nch, int C, int r) { return (int)((long)r * nch / C); }
// Dynamic shared memory: the P and W slices and the per-thread histogram.
inline size_t sample_smem_bytes(int V) {
  const int nch = sample_chunks(V), C = sample_ctas(V);
  const int per = (nch + C - 1) / C * kSampleChunk;
  return (size_t)(2 * per + (kSampleBins + 1) * kSampleThreads) * sizeof(float);
}

__device__ __forceinline__ uint4 philox_words(unsigned long long seed, uint32_t c0, uint32_t c1) {
  return philox4x32_10(make_uint4(c0, c1, 0u, 0u), (uint32_t)seed, (uint32_t)(seed >> 32));
}

// ------------------------------------------------ cluster helpers (PTX ISA 7.8+)
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Every thread of every CTA of the cluster; orders shared-memory writes before
// it against reads by any CTA after it.
__device__ __forceinline__ void cluster_barrier() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Load a float from CTA `rank`'s copy of a shared-memory variable.
__device__ __forceinline__ float ld_cluster(const float* p, uint32_t rank) {
  const uint32_t a = (uint32_t)__cvta_generic_to_shared(p);
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(rank));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(r) : "memory");
  return v;
}

// Every CTA's copy of one shared float, all loads issued before the first is
// used (one distributed-shared-memory round trip), in rank order.
__device__ __forceinline__ void ld_cluster_all(const float* p, int C, float (&v)[kSampleCtas]) {
#pragma unroll
  for (int r = 0; r < kSampleCtas; ++r) v[r] = r < C ? ld_cluster(p, (uint32_t)r) : 0.f;
}

struct SampleShared {
  float red[32 * 2];                 // warp partials of cluster reductions
  float xch[2][kSampleBins + 1];     // this CTA's values read by the cluster (double buffered)
  float tot[kSampleBins + 1];        // cluster totals
  float ctot[kSampleMaxChunks];      // this CTA's chunk totals
  float all[kSampleMaxChunks];       // every chunk total of the row
  float rem, gpick;
  int ch, tok, pick;
};

// Row-wide sum (or max) of NV per-thread values; every thread of every CTA
// returns the same totals. `ph` alternates the exchange buffer: a CTA writes
// buffer ph again only after the next barrier, which every reader of the
// previous use has passed after its reads.
template <int NV, bool MAX>
__device__ __forceinline__ void cl_reduce(float (&v)[NV], SampleShared& sh, int C, int& ph) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const float w = MAX ? warp_max(v[i]) : warp_sum(v[i]);
    if (lane == 0) sh.red[warp * NV + i] = w;
  }
  __syncthreads();
  if (threadIdx.x < NV) {
    float t = MAX ? -INFINITY : 0.f;
    for (int w = 0; w < nw; ++w) t = MAX ? fmaxf(t, sh.red[w * NV + threadIdx.x]) : t + sh.red[w * NV + threadIdx.x];
    sh.xch[ph][threadIdx.x] = t;
  }
  cluster_barrier();
  if (threadIdx.x < NV) {
    float t = MAX ? -INFINITY : 0.f, x[kSampleCtas];
    ld_cluster_all(&sh.xch[ph][threadIdx.x], C, x);
    for (int r = 0; r < C; ++r) t = MAX ? fmaxf(t, x[r]) : t + x[r];
    sh.tot[threadIdx.x] = t;
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < NV; ++i) v[i] = sh.tot[i];
  ph ^= 1;
}

// Online softmax partials (max m, sum of exp(x - m)) merged over the block
// and the cluster in a fixed order; every thread returns the row's (m, s).
__device__ __forceinline__ void sm_merge(float& m, float& s, float m2, float s2) {
  const float mx = fmaxf(m, m2);
  const float a = m == -INFINITY ? 0.f : s * expf(m - mx);
  const float b = m2 == -INFINITY ? 0.f : s2 * expf(m2 - mx);
  m = mx;
  s = a + b;
}

__device__ __forceinline__ void cl_softmax_stats(float& m, float& s, SampleShared& sh, int C, int& ph) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
    sm_merge(m, s, m2, s2);
  }
  if (lane == 0) {
    sh.red[warp * 2] = m;
    sh.red[warp * 2 + 1] = s;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float mm = -INFINITY, ss = 0.f;
    for (int w = 0; w < nw; ++w) sm_merge(mm, ss, sh.red[w * 2], sh.red[w * 2 + 1]);
    sh.xch[ph][0] = mm;
    sh.xch[ph][1] = ss;
  }
  cluster_barrier();
  if (threadIdx.x == 0) {
    float mm = -INFINITY, ss = 0.f, xm[kSampleCtas], xs[kSampleCtas];
    ld_cluster_all(&sh.xch[ph][0], C, xm);
    ld_cluster_all(&sh.xch[ph][1], C, xs);
    for (int r = 0; r < C; ++r) sm_merge(mm, ss, xm[r], xs[r]);
    sh.tot[0] = mm;
    sh.tot[1] = ss;
  }
  __syncthreads();
  m = sh.tot[0];
  s = sh.tot[1];
  ph ^= 1;
}

// Row-wide (max value, lowest index) over the cluster; every thread returns it.
__device__ __forceinline__ void am_merge(float& v, int& i, float v2, int i2) {
  if (v2 > v || (v2 == v && i2 < i)) {
    v = v2;
    i = i2;
  }
}

__device__ __forceinline__ void cl_argmax(float& v, int& i, SampleShared& sh, int C, int& ph) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
    am_merge(v, i, __shfl_xor_sync(0xffffffffu, v, o), __shfl_xor_sync(0xffffffffu, i, o));
  if (lane == 0) {
    sh.red[warp * 2] = v;
    sh.red[warp * 2 + 1] = __int_as_float(i);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int w = 0; w < nw; ++w) am_merge(bv, bi, sh.red[w * 2], __float_as_int(sh.red[w * 2 + 1]));
    sh.xch[ph][0] = bv;
    sh.xch[ph][1] = __int_as_float(bi);
  }
  cluster_barrier();
  if (threadIdx.x == 0) {
    float bv = -INFINITY, xv[kSampleCtas], xi[kSampleCtas];
    int bi = 0x7fffffff;
    ld_cluster_all(&sh.xch[ph][0], C, xv);
    ld_cluster_all(&sh.xch[ph][1], C, xi);
    for (int r = 0; r < C; ++r) am_merge(bv, bi, xv[r], __float_as_int(xi[r]));
    sh.tot[0] = bv;
    sh.tot[1] = __int_as_float(bi);
  }
  __syncthreads();
  v = sh.tot[0];
  i = __float_as_int(sh.tot[1]);
  ph ^= 1;
}

// Row loops visit E consecutive elements per step (E = 4 when V % 4 == 0: one
// 16-byte load or store per step, else 1): thread tid takes steps tid,
// tid + blockDim.x, ... and, within a step, elements in index order.
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

// Largest bit pattern v with F(v) >= target, F(v) = sum (or count) of the
// row's elements >= v (p <= 1 for every element, so [0, 2^30) brackets every
// pattern). Each pass histograms this CTA's slice over 32 bins of width 2^s
// starting at lo plus one bin above (per-thread columns of `hist`, summed in
// a fixed order), adds the cluster's bins, and keeps the highest bin whose
// suffix sum reaches the target; s goes 25, 20, ..., 5, 0. `at_cut` receives
// F at the result (the last pass's suffix sum of bins of width 1).
template <bool COUNT, int E>
__device__ float cl_cutoff(const float* P, int n, float target, float* hist, SampleShared& sh, int C,
                           int& ph, float* at_cut) {
  const int tid = threadIdx.x, nt = blockDim.x, lane = tid & 31, warp = tid >> 5, nw = nt >> 5;
  uint32_t lo = 0u;
  int s = 30 - kSampleBinShift;
  for (;;) {
#pragma unroll
    for (int i = 0; i <= kSampleBins; ++i) hist[i * nt + tid] = 0.f;
    for (int j = tid; j < n / E; j += nt) {
      const Vf<E> x = ldv<E>(P, j);
#pragma unroll
      for (int i = 0; i < E; ++i) {
        const uint32_t b = __float_as_uint(x.v[i]);
        if (b >= lo) {
          const uint32_t d = min((b - lo) >> s, (uint32_t)kSampleBins);
          hist[d * nt + tid] += COUNT ? 1.f : x.v[i];
        }
      }
    }
    __syncthreads();
    for (int bin = warp; bin <= kSampleBins; bin += nw) {
      float t = 0.f;
      for (int j = lane; j < nt; j += 32) t += hist[bin * nt + j];
      t = warp_sum(t);
      if (lane == 0) sh.xch[ph][bin] = t;
    }
    cluster_barrier();
    if (tid <= kSampleBins) {
      float t = 0.f, x[kSampleCtas];
      ld_cluster_all(&sh.xch[ph][tid], C, x);
      for (int r = 0; r < C; ++r) t += x[r];
      sh.tot[tid] = t;
    }
    __syncthreads();
    ph ^= 1;
    if (warp == 0) {
      // suffix sums G[i] = above + sum_{j >= i} bin[j] (a fixed shuffle tree),
      // and the highest bin whose G reaches the target (bin 0 if none)
      static_assert(kSampleBins == 32, "one bin per lane");
      float v = sh.tot[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_down_sync(0xffffffffu, v, o);
        if (lane + o < 32) v += y;
      }
      v += sh.tot[kSampleBins];
      const unsigned ok = __ballot_sync(0xffffffffu, v >= target);
      const int pk = ok ? 31 - __clz(ok) : 0;
      const float gk = __shfl_sync(0xffffffffu, v, pk);
      if (lane == 0) {
        sh.pick = pk;
        sh.gpick = gk;
      }
    }
    __syncthreads();
    const int pick = sh.pick;
    const float g = sh.gpick;
    lo += (uint32_t)pick << s;
    if (s == 0) {
      *at_cut = g;
      break;
    }
    s = s >= kSampleBinShift ? s - kSampleBinShift : 0;
  }
  return __uint_as_float(lo);
}

// Inverse-CDF draw from non-negative weights w (need not be normalised) over
// the whole row: target = u * total; the first 2048-chunk whose inclusive CDF
// exceeds target, then the first token of it whose inclusive CDF exceeds
// target - preceding mass.
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

// Total of local chunk lc of a slice of n elements.
__device__ __forceinline__ float chunk_total(const float* w, int lc, int n) {
  const int lane = threadIdx.x & 31;
  float tot = 0.f;
  for (int i0 = 0; i0 < kSampleChunk / 32; i0 += 8) {
    float x[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int t = lc * kSampleChunk + (i0 + j) * 32 + lane;
      x[j] = t < n ? w[t] : 0.f;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) tot += __shfl_sync(0xffffffffu, warp_incl_scan(x[j]), 31);
  }
  return tot;
}

// Returns the drawn token in the CTA that owns its chunk and -1 in the others.
// w: this CTA's slice (chunks [c0, c1), n elements).
__device__ int cl_pick(const float* w, int n, int c0, int c1, int nch, int C, float u, SampleShared& sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int c = c0 + warp; c < c1; c += nw) {          // one warp per chunk
    const float a = chunk_total(w, c - c0, n);
    if (lane == 0) sh.ctot[c - c0] = a;
  }
  cluster_barrier();
  if ((int)threadIdx.x < nch) {
    const int c = threadIdx.x;
    int r = 0;
    while (r + 1 < C && sample_chunk0(nch, C, r + 1) <= c) ++r;
    sh.all[c] = ld_cluster(&sh.ctot[c - sample_chunk0(nch, C, r)], (uint32_t)r);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float total = 0.f;
    for (int c = 0; c < nch; ++c) total += sh.all[c];
    const float target = u * total;
    float cdf = 0.f, pre = 0.f;
    int ch = -1;
    for (int c = 0; c < nch; ++c) {
      if (cdf + sh.all[c] > target) {
        ch = c;
        pre = cdf;
        break;
      }
      cdf += sh.all[c];
    }
    if (ch < 0) {
      ch = 0;
      pre = 0.f;
    }
    sh.ch = ch;
    sh.rem = target - pre;
  }
  __syncthreads();
  const int ch = sh.ch;
  const float rem = sh.rem;
  if (ch < c0 || ch >= c1) return -1;
  const int lc = ch - c0;
  if (warp == 0) {
    int found = -1;                                  // nothing exceeds: first token of the chunk
    float pre = 0.f;
    for (int i0 = 0; i0 < kSampleChunk / 32 && found < 0; i0 += 8) {
      float x[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int t = lc * kSampleChunk + (i0 + j) * 32 + lane;
        x[j] = t < n ? w[t] : 0.f;
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
    if (lane == 0) sh.tok = found >= 0 ? found : ch * kSampleChunk;
  }
  __syncthreads();
  return sh.tok;
}

__device__ __forceinline__ void put_decision(long long* d, long long t, long long a, long long b, long long c,
                                             long long e) {
  d[0] = t;
  d[1] = a;
  d[2] = b;
  d[3] = c;
  d[4] = e;
}

// grid = rows x C CTAs, cluster (C, 1, 1), kSampleThreads threads,
// sample_smem_bytes(V) of dynamic shared memory.
template <int E>
__global__ void __launch_bounds__(kSampleThreads) sample_kernel(SampleArgs a) {
  pdl_launch_dependents();
  pdl_wait();
  extern __shared__ __align__(16) float s_dyn[];
  __shared__ SampleShared sh;
  const int V = a.V, nch = sample_chunks(V), C = sample_ctas(V);
  const int rank = (int)cluster_rank();
  const int row = blockIdx.x / C;
  const int mrow = a.meta_row0 + row;
  // every CTA of a cluster reads the same metadata, so these exits are
  // cluster-uniform and come before the first cluster barrier
  if (a.meta.get(kMetaPos, mrow) < 0) return;   // inactive lane
  const int rq = a.meta.get(kMetaReq, mrow);
  if (rq < 0 || rq >= a.n_params) {
    if (rank == 0 && threadIdx.x == 0) atomicExch(a.err, kDevBadIndex);
    return;
  }
  const SampleParams prm = a.params[rq];
  const int kind = a.meta.get(kMetaKind, mrow);
  const int first = a.meta.get(kMetaFirst, mrow);
  const int second = a.meta.get(kMetaSecond, mrow);
  const int slot = a.meta.get(kMetaStateIn, mrow);
  const uint32_t cycle = (uint32_t)a.meta.get(kMetaCycle, mrow);
  const bool need_bank = kind == 0 || kind == 1 || first >= 0;
  if ((need_bank && (slot < 0 || slot >= a.bank_rows)) || first >= V || second >= V ||
      (kind == 1 && first < 0)) {
    if (rank == 0 && threadIdx.x == 0) atomicExch(a.err, kDevBadIndex);
    return;
  }
  const int c0 = sample_chunk0(nch, C, rank), c1 = sample_chunk0(nch, C, rank + 1);
  const int n0 = c0 * kSampleChunk;
  const int n = min(c1 * kSampleChunk, V) - n0;
  const int per = (nch + C - 1) / C * kSampleChunk;
  float* P = s_dyn;
  float* W = s_dyn + per;
  float* hist = s_dyn + 2 * per;
  const float* lg_row = a.logits + (long)row * V;
  const float* lg = lg_row + n0;
  long long* dec = a.decisions + (long)row * 5;
  int ph = 0;
  const int NV = n / E, tid = threadIdx.x, nt = blockDim.x;

  if (prm.top_k == 1) {   // greedy row: argmax, the lowest index on ties
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int j = tid; j < NV; j += nt) {
      const Vf<E> x = ldv<E>(lg, j);
#pragma unroll
      for (int i = 0; i < E; ++i)
        if (x.v[i] > bv) {   // indices increase within a thread, so ties keep the lower
          bv = x.v[i];
          bi = n0 + j * E + i;
        }
    }
    cl_argmax(bv, bi, sh, C, ph);
    if (rank == 0 && threadIdx.x == 0) put_decision(dec, bi == 0x7fffffff ? 0 : bi, 0, 0, 0, 0);
    cluster_barrier();   // no CTA leaves while another may still read its shared memory
    return;
  }

  // softmax(logits / T) in fp32: online (max, sum) per thread, merged over
  // the row, then P = exp(x / T - max) / sum
  const float invT = 1.f / prm.temperature;
  float mx = -INFINITY, sm = 0.f;
#pragma unroll 4
  for (int j = tid; j < NV; j += nt) {
    const Vf<E> x = ldv<E>(lg, j);
#pragma unroll
    for (int i = 0; i < E; ++i) {
      const float y = x.v[i] * invT;
      if (y > mx) {
        sm = mx == -INFINITY ? 0.f : sm * expf(mx - y);
        mx = y;
      }
      sm += expf(y - mx);
    }
  }
  cl_softmax_stats(mx, sm, sh, C, ph);
#pragma unroll 4
  for (int j = tid; j < NV; j += nt) {
    Vf<E> x = ldv<E>(lg, j);
#pragma unroll
    for (int i = 0; i < E; ++i) x.v[i] = expf(fmaf(x.v[i], invT, -mx)) / sm;
    stv<E>(P, j, x);
  }
  __syncthreads();
  // top-k / top-p cutoffs, then renormalise over the kept support
  const int k = prm.top_k >= V ? 0 : prm.top_k;
  const bool cutting = k > 0 || prm.top_p < 1.f;
  float cut = 0.f, kept[1] = {1.f};
  if (cutting) {
    float mass_p = 0.f, count_k = 0.f;
    if (prm.top_p < 1.f) cut = cl_cutoff<false, E>(P, n, prm.top_p, hist, sh, C, ph, &mass_p);
    if (k > 0) {
      const float ck = cl_cutoff<true, E>(P, n, (float)k, hist, sh, C, ph, &count_k);
      cut = prm.top_p < 1.f ? fmaxf(cut, ck) : ck;
    }
    if (k == 0) {
      kept[0] = mass_p;   // the top-p pass summed exactly the elements >= cut
    } else {
      kept[0] = 0.f;
#pragma unroll 4
      for (int j = tid; j < NV; j += nt) {
        const Vf<E> x = ldv<E>(P, j);
#pragma unroll
        for (int i = 0; i < E; ++i) kept[0] += x.v[i] >= cut ? x.v[i] : 0.f;
      }
      cl_reduce<1, false>(kept, sh, C, ph);
    }
#pragma unroll 4
    for (int j = tid; j < NV; j += nt) {
      Vf<E> x = ldv<E>(P, j);
#pragma unroll
      for (int i = 0; i < E; ++i) {
        x.v[i] = x.v[i] >= cut ? x.v[i] : 0.f;
        x.v[i] = x.v[i] / kept[0];
      }
      stv<E>(P, j, x);
    }
  }
  __syncthreads();
  // P of one token, by the slice loops' operations (same bits in every CTA)
  auto prob = [&](int t) {
    float p = expf(fmaf(lg_row[t], invT, -mx)) / sm;
    if (cutting) {
      p = p >= cut ? p : 0.f;
      p = p / kept[0];
    }
    return p;
  };

  // the request's stream: its seed, cycle counter and readout row
  const unsigned long long seed = (unsigned long long)(uint32_t)a.meta.get(kMetaSeedLo, mrow) |
                                  ((unsigned long long)(uint32_t)a.meta.get(kMetaSeedHi, mrow) << 32);
  const uint32_t draw_row = (uint32_t)a.meta.get(kMetaDrawRow, mrow);
  const uint4 w4 = philox_words(seed, cycle, draw_row);
  const float u0 = (float)(w4.x >> 8) * (1.f / 16777216.f);
  const float u1 = (float)(w4.y >> 8) * (1.f / 16777216.f);
  const float u2 = (float)(w4.z >> 8) * (1.f / 16777216.f);
  const bool lead = threadIdx.x == 0;

  if (kind == 0) {                                     // q1: draw and keep P
    float* q1 = a.q1_bank + (long)slot * V + n0;
#pragma unroll 4
    for (int j = tid; j < NV; j += nt) stv<E>(q1, j, ldv<E>(P, j));
    const int x = cl_pick(P, n, c0, c1, nch, C, u0, sh);
    if (x >= 0 && lead) put_decision(dec, x, 1, 0, 0, 0);
  } else if (kind == 1) {                              // q2: conditional residual
    const float* q1 = a.q1_bank + (long)slot * V;
    float mass[1] = {0.f};
#pragma unroll 4
    for (int j = tid; j < NV; j += nt) {
      const Vf<E> p = ldv<E>(P, j), q = ldv<E>(q1 + n0, j);
      Vf<E> r;
#pragma unroll
      for (int i = 0; i < E; ++i) {
        r.v[i] = n0 + j * E + i == first ? 0.f : fmaxf(p.v[i] - q.v[i], 0.f);
        mass[0] += r.v[i];
      }
      stv<E>(W, j, r);
    }
    cl_reduce<1, false>(mass, sh, C, ph);
    float* R = a.r_bank + (long)slot * V + n0;
#pragma unroll 4
    for (int j = tid; j < NV; j += nt) {
      Vf<E> r = ldv<E>(W, j);
#pragma unroll
      for (int i = 0; i < E; ++i) r.v[i] = mass[0] > 0.f ? r.v[i] / mass[0] : 0.f;
      stv<E>(R, j, r);
    }
    const bool action = mass[0] > 0.f && prob(first) < q1[first];
    const int y = cl_pick(W, n, c0, c1, nch, C, u0, sh);
    if (y >= 0 && lead) put_decision(dec, action ? y : first, action, action, 0, 0);
  } else if (first < 0) {                              // final without a proposal
    const int x = cl_pick(P, n, c0, c1, nch, C, u0, sh);
    if (x >= 0 && lead) put_decision(dec, x, 0, 0, 0, 0);
  } else {                                             // final verification
    const float* q1 = a.q1_bank + (long)slot * V;
    const float acc = fminf(1.f, prob(first) / q1[first]);
    if (u0 < acc) {
      if (rank == 0 && lead) put_decision(dec, first, 0, 1, 0, 0);
    } else {
      float mFP[2] = {0.f, 0.f};
#pragma unroll 4
      for (int j = tid; j < NV; j += nt) {
        const Vf<E> p = ldv<E>(P, j), q = ldv<E>(q1 + n0, j);
        Vf<E> f;
#pragma unroll
        for (int i = 0; i < E; ++i) {
          f.v[i] = fmaxf(p.v[i] - q.v[i], 0.f);
          mFP[0] += f.v[i];
          mFP[1] += p.v[i];
        }
        stv<E>(W, j, f);
      }
      cl_reduce<2, false>(mFP, sh, C, ph);
      const float mF = mFP[0], mP = mFP[1];
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
        const float ps = prob(second);
        const float fs = mF > 0.f ? fmaxf(ps - q1[second], 0.f) / mF : ps / (mP > 0.f ? mP : 1.f);
        acc2 = u1 < fminf(1.f, fs / R[second]);
        float mG[1] = {0.f};
#pragma unroll 4
        for (int j = tid; j < NV; j += nt) {
          const Vf<E> f = ldv<E>(W, j), r = ldv<E>(R + n0, j);
#pragma unroll
          for (int i = 0; i < E; ++i) mG[0] += fmaxf(f.v[i] - r.v[i], 0.f);
        }
        cl_reduce<1, false>(mG, sh, C, ph);
        if (mG[0] > 0.f) {
#pragma unroll 4
          for (int j = tid; j < NV; j += nt) {
            Vf<E> f = ldv<E>(W, j);
            const Vf<E> r = ldv<E>(R + n0, j);
#pragma unroll
            for (int i = 0; i < E; ++i) f.v[i] = fmaxf(f.v[i] - r.v[i], 0.f) / mG[0];
            stv<E>(W, j, f);
          }
        }
        __syncthreads();
      }
      if (acc2) {
        if (rank == 0 && lead) put_decision(dec, second, 0, 2, 1, 0);
      } else {
        const int x = cl_pick(W, n, c0, c1, nch, C, u2, sh);
        if (x >= 0 && lead) put_decision(dec, x, 0, 0, 1, second >= 0);
      }
    }
  }
  // no CTA leaves while another may still read its shared memory
  cluster_barrier();
}

}  // namespace ls
