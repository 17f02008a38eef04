// Persistent stack kernel: one launch runs a whole role call -- the timeline
// mapping update, the input gather / norm, and every decoder layer's GEMMs,
// attention and residual rows -- on one CTA per SM.
//
// Why: a decode role call is a chain of ~7 dependent steps per layer, each
// moving 8-50 MB. As separate kernels every step pays launch, ramp-up and
// drain (about 4 us each), and the GPU streams weights at under half of HBM
// bandwidth. Here the steps become phases of one program. Phases are
// separated by a grid-wide arrival counter, and the weight stream never
// waits for them: the TMA producer of each CTA walks its whole list of weight
// tiles, across phases and layers, and keeps its shared-memory ring full.
// Only the (small) activation tile of a ring stage waits for the phase that
// produces it.
//
// CTA layout (256 threads):
//   warp 0      TMA producer (one thread): weight boxes ahead of the phase
//               barrier, activation boxes once the producing phase completed
//   warp 1      MMA issuer (one thread): tcgen05.mma into one of two TMEM
//               accumulators (BN fp32 columns each)
//   warps 2..7  workers (192 threads): GEMM epilogues (warps 4..7 read TMEM,
//               one 32-lane quadrant each), attention, per-lane rows
//
// GEMM phases are split "stream-K" style: the phase's (tile, k-block) space,
// T = m_tiles * KB, is cut into Gw = min(grid, T) equal contiguous ranges,
// one per CTA. A range covers the end of one tile, whole tiles, and the start
// of another; each piece is a segment. A CTA writes each segment's partial
// tile to one of two slots it owns (slot 0: its first segment, slot 1: the
// others, used in order). The last contributor of a tile (atomic ticket)
// sums the contributors' partials in CTA order and applies the epilogue. Cut
// points depend only on (M, K, grid), never on the lanes, so a lane's result
// does not depend on the batch it runs in.
//
// Ordering is dataflow, not phase barriers. Each unit of work publishes a
// completion counter after its writes (a GEMM tile, an attention (lane, kv
// head) merge, a per-lane row), and each consumer waits only for the counters
// of what it reads: attention for kv head g waits for the QKV tiles holding
// g's q, k, v rows; an O-projection activation box for the heads it covers; a
// down-projection box for the one gate/up tile that produced it; a row for
// all tiles of its GEMM. Every buffer reuse is ordered through these chains
// (a GEMM phase transitively waits for all tiles of the GEMM two before it),
// so partial slots and tile tickets alternate between two sets by GEMM parity.
// All CTAs must be co-resident (one per SM, checked by a start counter with a
// bounded wait). Every wait is bounded: on timeout the CTA records an error,
// stops issuing work, waits for its own copies and MMAs in flight, frees its
// TMEM and exits; other CTAs see the error word and exit too. The last CTA to
// exit zeroes the counters for the next launch.
#pragma once

#include "common.cuh"
#include "gemm_tc.cuh"
#include "stack_api.cuh"

namespace ls {

template <int BN, int ST>
struct StkSmem {
  static constexpr int kSubA = kGemmBM * kGemmBK * 2;   // one 128 x 64 weight sub-tile
  static constexpr int kSubB = BN * kGemmBK * 2;         // one BN x 64 activation sub-tile
  static constexpr int kA = kSubA * kStkSub;
  static constexpr int kB = kSubB * kStkSub;
  static constexpr int kStage = kA + kB;
  static constexpr int kRing = ST * kStage;
  static constexpr int kWork = 12288;           // worker scratch
  static constexpr int kBars = (2 * ST + 5) * 8;
  static constexpr int kTotal = 1024 + kRing + kWork + kBars;
  static constexpr uint32_t kTmemCols = 2 * BN < 32 ? 32 : 2 * BN;
  static_assert(kStage % 1024 == 0, "ring stages must keep 1024-byte alignment");
  static_assert(kTotal <= 232448, "shared memory above the sm_100 per-block limit");
};

// ------------------------------------------------------------------ helpers
__device__ __forceinline__ bool mbar_test(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

__device__ __forceinline__ void named_bar(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

__device__ __forceinline__ float4 f4_add(float4 a, float4 b) {
  return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
}


__device__ __forceinline__ void stk_trace(const StackParams& P, int phase, int field) {
  if (P.trace) P.trace[((long)phase * gridDim.x + blockIdx.x) * kStkTraceFields + field] = gtime_ns();
}

// CTA 0's per-stage event log after the phase table (trace runs only):
// [4][kStkLogMax] SM clocks of weight issue, activation issue, MMA take of
// ring stage i, and of the input-frontier fences (by fence count).
constexpr int kStkLogMax = 4096;
__device__ __forceinline__ void stk_log(const StackParams& P, int kind, long long i) {
  if (P.trace && blockIdx.x == 0 && i < kStkLogMax)
    P.trace[(long)(P.n_phases + 1) * gridDim.x * kStkTraceFields + kind * kStkLogMax + i] =
        (unsigned long long)clock64();
}

__device__ __forceinline__ void stk_trace_value(const StackParams& P, int phase, int field,
                                                unsigned long long v) {
  if (P.trace) P.trace[((long)phase * gridDim.x + blockIdx.x) * kStkTraceFields + field] = v;
}

// Time-bounded mbarrier wait that gives up early once the CTA is aborting or
// another CTA has recorded an error.
__device__ __forceinline__ bool stk_wait(uint32_t bar, uint32_t parity, volatile int* abort_, int* err,
                                         int code) {
  const unsigned long long t0 = gtime_ns();
  for (uint32_t i = 0;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63u) == 63u) {
      if (*abort_ || ld_volatile(err) != 0) break;
      if (gtime_ns() - t0 > kStkWaitNs) {
        atomicExch(err, code);
        break;
      }
    }
  }
  *abort_ = 1;
  return false;
}

// Time-bounded wait for copies or MMAs already issued (used on exit paths).
__device__ __forceinline__ void stk_drain(uint32_t bar, uint32_t parity) {
  const unsigned long long t0 = gtime_ns();
  while (!mbar_try_wait(bar, parity))
    if (gtime_ns() - t0 > kStkWaitNs) return;
}

__device__ __forceinline__ unsigned ld_relaxed(const unsigned* p) {
  unsigned v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void fence_acquire_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }

__device__ __forceinline__ int ld_acquire_s32(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Counter update with release semantics (cumulative over the writes of the
// threads that synchronised with this one through a CTA barrier).
__device__ __forceinline__ void red_release_add(int* p, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ int atom_acq_rel_add(int* p, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

// Activations of decode widths (BN <= 32, up to 16 lanes) are copied into the
// ring by a warp with L2 loads (generic proxy); wider calls use TMA boxes.
template <int BN>
struct ActPath {
  static constexpr bool kLdg = BN <= 32;
};

// Time-bounded wait until *ctr >= target, with acquire semantics on success
// (relaxed polls, then a fence). Gives up when another CTA has recorded an
// error (checked every 16 polls) or after limit_ns.
__device__ __forceinline__ bool grid_wait(const unsigned* ctr, unsigned target, volatile int* abort_,
                                          int* err, int code, unsigned long long limit_ns) {
  const unsigned long long t0 = gtime_ns();
  for (uint32_t i = 0;; ++i) {
    if (ld_relaxed(ctr) >= target) {
      ld_acquire(ctr);   // acquire (the counter only grows)
      return true;
    }
    if ((i & 15u) == 15u) {
      if (*abort_ || ld_volatile(err) != 0) break;
      if (gtime_ns() - t0 > limit_ns) {
        if (ld_acquire(ctr) >= target) return true;
        atomicExch(err, code);
        break;
      }
    }
    __nanosleep(kStkPollNs);   // back off: many CTAs poll the same few lines
  }
  *abort_ = 1;
  return false;
}

// Sum over the 192 worker threads; `red` holds 8 floats. Fixed order.
__device__ __forceinline__ float worker_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, w = (threadIdx.x >> 5) - kStkWorkerTid0 / 32;
  v = warp_sum(v);
  named_bar(kBarWorkers, kStkWorkers);
  if (lane == 0) red[w] = v;
  named_bar(kBarWorkers, kStkWorkers);
  float t = lane < 6 ? red[lane] : 0.f;
  return warp_sum(t);
}

// Completion target of a phase-level dependency.
__device__ __forceinline__ int dep_tot_target(const StackParams& P, int kind, int q) {
  return kind == kDepTotLanes ? P.n : kind == kDepTotTiles ? P.phases[q].m_tiles : 0;
}

// One thread: wait for the phase-level (tot) dependencies of `ph`.
__device__ __forceinline__ bool wait_tot_deps(const StackParams& P, const Phase& ph, volatile int* abort_) {
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int k = ph.dep_kind[i];
    if (k != kDepTotLanes && k != kDepTotTiles) continue;
    const int q = ph.dep_phase[i];
    if (!grid_wait(reinterpret_cast<const unsigned*>(P.tot + q), (unsigned)dep_tot_target(P, k, q), abort_,
                   P.err, kDevTimeoutGrid, kStkWaitNs))
      return false;
  }
  return true;
}

// Publish work done by the 192 workers (or the 128 epilogue threads, `nthreads`):
// after a CTA barrier one thread adds to the counters with release semantics,
// which covers the barrier's participants' writes. `proxy`: the outputs are
// read by TMA (async proxy), so each writer also fences its writes for it.
__device__ __forceinline__ void publish(int bar, int nthreads, bool leader, int* c1, int* c2, bool proxy) {
  if (proxy) fence_proxy_async_global();   // consumers read through TMA
  named_bar(bar, nthreads);
  if (leader) {
    if (c1) red_release_add(c1, 1);
    if (c2) red_release_add(c2, 1);
  }
}

// This CTA's k-block range of a GEMM phase (empty if it takes no part).
struct KRange {
  int lo, hi, T, Gw;
};

__device__ __forceinline__ KRange gemm_range(const Phase& ph) {
  KRange r;
  r.T = ph.m_tiles * ph.KB;
  r.Gw = min((int)gridDim.x, r.T);
  const int c = blockIdx.x;
  if (c >= r.Gw) {
    r.lo = r.hi = 0;
  } else {
    r.lo = (int)((long)c * r.T / r.Gw);
    r.hi = (int)((long)(c + 1) * r.T / r.Gw);
  }
  return r;
}

// CTAs whose ranges overlap tile t: [first, last].
__device__ __forceinline__ int2 tile_ctas(int t, int KB, int T, int Gw) {
  const long a = (long)t * KB, b = (long)(t + 1) * KB;
  const int cf = (int)(((a + 1) * Gw + T - 1) / T) - 1;
  const int cl = (int)((b * Gw + T - 1) / T) - 1;
  return make_int2(cf, cl);
}

// Walks a CTA's k-blocks across all GEMM phases of the program, in order,
// keeping the current phase's fields in registers.
struct KbIter {
  int p, f, lo, hi;
  int KB, epi, xbuf, head, wmap;
  int dep_kind[2], dep_off[2], dep_target[2];   // activation inputs (counter index, target)
  int dep_kdim[2];                              // K of this GEMM (bounds a unit's columns)
  __device__ __forceinline__ void seek(const StackParams& P, int from) {
    for (p = from; p < P.n_phases; ++p) {
      const Phase& ph = P.phases[p];
      if (ph.kind != kPhGemm) continue;
      const KRange r = gemm_range(ph);
      if (r.lo < r.hi) {
        f = lo = r.lo;
        hi = r.hi;
        KB = ph.KB;
        epi = ph.epi;
        xbuf = ph.xbuf;
        head = ph.head;
        wmap = ph.wmap;
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const int k = ph.dep_kind[i], q = ph.dep_phase[i];
          dep_kind[i] = k;
          dep_kdim[i] = ph.K;
          if (k == kDepTotLanes || k == kDepTotTiles) {
            dep_off[i] = q;
            dep_target[i] = dep_tot_target(P, k, q);
          } else if (k == kDepKbHead || k == kDepKbTile) {
            dep_off[i] = P.phases[q].cnt_off;
            dep_target[i] = k == kDepKbHead ? P.n : 1;
          } else {
            dep_off[i] = 0;
            dep_target[i] = 0;
          }
        }
        return;
      }
    }
  }
  __device__ __forceinline__ bool valid(const StackParams& P) const { return p < P.n_phases; }
  __device__ __forceinline__ void step(const StackParams& P) {
    if (++f == hi) seek(P, p + 1);
  }
};

// Inputs of k-unit f (columns [u * kStkBK, +kStkBK) of the GEMM's K) that are
// produced piecewise: the attention kv heads covering those columns (O
// projection), or the two 64-column gate/up tiles that wrote them (down
// projection). ACQ: acquire loads; else relaxed (the caller fences).
template <bool ACQ>
__device__ __forceinline__ bool unit_inputs_ready(const StackParams& P, const KbIter& a, int f, int G) {
  const int c0 = (f % a.KB) * kStkBK;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int k = a.dep_kind[i];
    int lo, hi;
    if (k == kDepKbHead) {
      const int qd = P.NH * P.HD;
      lo = c0 / (P.HD * G);
      hi = (min(c0 + kStkBK, qd) - 1) / (P.HD * G);
    } else if (k == kDepKbTile) {
      lo = c0 / kGemmBK;
      hi = (min(c0 + kStkBK, a.dep_kdim[i]) - 1) / kGemmBK;
    } else {
      continue;
    }
    for (int x = lo; x <= hi; ++x) {
      const int* c = P.cnt + a.dep_off[i] + x;
      const int v = ACQ ? ld_acquire_s32(c) : (int)ld_relaxed(reinterpret_cast<const unsigned*>(c));
      if (v < a.dep_target[i]) return false;
    }
  }
  return true;
}

// ----------------------------------------------------------- TMA producers
// Weights (warp 0): walk the CTA's k-blocks across all GEMM phases and issue
// each weight box as soon as its ring stage is free -- weights never depend on
// earlier phases, so the ring fills ahead across phase barriers. Posting the
// stage's expect_tx (weight + activation bytes) precedes the count s_iw.
// Activations (warp 8): trail the weights; issue stage i's activation box
// once i < s_iw and every phase before the stage's GEMM phase has completed
// on all CTAs. Two threads, so a phase's activation boxes go out in a burst
// when its inputs are ready instead of interleaved with weight issues.
template <int BN, int ST>
__device__ void stk_weights(const StackLaunch& L, uint8_t* smem, uint32_t full0, uint32_t empty0,
                            volatile int* abort_, volatile long long* s_iw, volatile int* s_wdone) {
  using S = StkSmem<BN, ST>;
  const StackParams& P = L.P;
  KbIter w;
  w.seek(P, 0);
  long long iw = 0;
  int s = 0;
  uint32_t use = 0;   // how many times stage s has been filled before
  while (w.valid(P)) {
    if (use > 0 && !stk_wait(empty0 + 8 * s, (use - 1) & 1, abort_, P.err, kDevTimeoutEmpty)) break;
    const uint32_t fb = full0 + 8 * s;
    mbar_expect_tx(fb, ActPath<BN>::kLdg ? S::kA : S::kStage);   // weights (+ a TMA activation box)
    const int t = w.f / w.KB, kc0 = (w.f % w.KB) * kStkBK;
    const CUtensorMap* wm = &L.wmap[w.wmap];
#pragma unroll
    for (int u = 0; u < kStkSub; ++u) {
      const uint32_t dst = smem_u32(smem + s * S::kStage + u * S::kSubA);
      const int kc = kc0 + u * kGemmBK;   // past K: the box reads the zero fill
      if (w.epi == kEpiSwiGLU) {
        // 64 gate rows and the matching 64 up rows
        tma_load_2d(dst, wm, fb, kc, t * (kGemmBM / 2));
        tma_load_2d(dst + kGemmBM / 2 * kGemmBK * 2, wm, fb, kc, P.I + t * (kGemmBM / 2));
      } else {
        tma_load_2d(dst, wm, fb, kc, t * kGemmBM);
      }
    }
    stk_log(P, 0, iw);
    w.step(P);
    ++iw;
    *s_iw = iw;
    if (++s == ST) {
      s = 0;
      ++use;
    }
  }
  __threadfence_block();   // the final count is visible before the done flag
  *s_wdone = 1;
}

template <int BN, int ST>
__device__ void stk_acts(const StackLaunch& L, uint8_t* smem, uint32_t full0, volatile int* abort_,
                         volatile long long* s_iw, volatile int* s_wdone) {
  using S = StkSmem<BN, ST>;
  const StackParams& P = L.P;
  KbIter a;
  a.seek(P, 0);
  long long ia = 0;
  bool waited = false;     // griddepcontrol.wait done
  uint32_t polls = 0;
  const int G = P.NH / P.NKV;
  const int head_row0 = 2 * P.head_lane0;
  int sa = 0;   // ring stage of activation ia
  auto issue = [&]() {
#pragma unroll
    for (int u = 0; u < kStkSub; ++u)
      tma_load_2d(smem_u32(smem + sa * S::kStage + S::kA + u * S::kSubB), &L.xmap[a.xbuf],
                  full0 + 8 * (uint32_t)sa, (a.f % a.KB) * kStkBK + u * kGemmBK, a.head ? head_row0 : 0);
    stk_log(P, 1, ia);
    a.step(P);
    ++ia;
    if (++sa == ST) sa = 0;
  };
  long long n_fences = 0;
  // Inputs are known complete for the stages of phase known_p below f = known_f.
  // A check extends that frontier over up to 8 k-blocks at once, and only an
  // extension pays the acquire and proxy fences.
  int known_p = -1, known_f = 0;
  auto kb_ready = [&](int f) -> bool { return unit_inputs_ready<false>(P, a, f, G); };
  auto inputs_ready = [&]() -> bool {   // true: the stage at a.f may load (fences done)
    if (known_p == a.p && a.f < known_f) return true;
    if (known_p != a.p) {
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int k = a.dep_kind[i];
        if ((k == kDepTotLanes || k == kDepTotTiles) &&
            (int)ld_relaxed(reinterpret_cast<const unsigned*>(P.tot + a.dep_off[i])) < a.dep_target[i])
          return false;
      }
      known_p = a.p;
      known_f = a.f;
    }
    int f = known_f;
    const int lim = min(a.hi, known_f + 8);
    while (f < lim && kb_ready(f)) ++f;
    if (f == known_f) return false;
    known_f = f;
    fence_acquire_gpu();
    fence_proxy_async_global();            // generic writes of the producers -> TMA reads
    stk_log(P, 3, n_fences++);
    return true;
  };
  unsigned long long idle_since = 0;
  uint32_t idles = 0;
  auto idle = [&]() -> bool {   // false: give up
    if (*abort_) return false;
    __nanosleep(kStkPollNs);
    if ((++idles & 63u) != 0) return true;
    const unsigned long long now = gtime_ns();
    if (idle_since == 0) idle_since = now;
    if (now - idle_since > kStkWaitNs) {
      atomicExch(P.err, kDevTimeoutGrid);
      *abort_ = 1;
      return false;
    }
    return true;
  };
  while (a.valid(P)) {
    if (ia >= *s_iw) {                       // this stage's weight box not issued yet
      if (*s_wdone) {
        // the weight thread stored its last count before the done flag:
        // re-read the count now that the flag is seen
        if (ia < *s_iw) continue;
        *abort_ = 1;                         // weights stopped early: aborting
        break;
      }
      if (!idle()) break;
      continue;
    }
    if (!waited) {
      pdl_wait();
      waited = true;
    }
    if (!inputs_ready()) {
      if ((++polls & 15u) == 0 && ld_volatile(P.err) != 0) {
        *abort_ = 1;
        break;
      }
      if (!idle()) break;
      continue;
    }
    if (P.trace && a.f == a.lo) {
      stk_trace(P, a.p, 6);
      stk_trace_value(P, a.p, 11, (unsigned long long)min((long long)(a.hi - a.f), *s_iw - ia));
    }
    idle_since = 0;
    idles = 0;
    if (P.trace && a.f == a.lo) stk_trace(P, a.p, 3);
    if (P.trace && a.f + 1 == a.hi) stk_trace(P, a.p, 8);
    issue();
  }
  // Exit. Normally every activation box has been issued here. When aborting,
  // give every stage whose weight box was issued its activation box (the load
  // reads in-bounds memory; the results are discarded). Then wait until all
  // boxes have landed so that no copy completes after the CTA exits.
  const unsigned long long t0 = gtime_ns();
  while (!*s_wdone && gtime_ns() - t0 < kStkWaitNs) __nanosleep(64);
  const long long iw = *s_iw;
  if (ia < iw && a.valid(P)) {
    *abort_ = 1;
    if (ld_volatile(P.err) == 0) atomicExch(P.err, kDevTimeoutGrid);
    while (ia < iw && a.valid(P)) issue();
  }
  for (long long i = iw > ST ? iw - ST : 0; i < iw; ++i)
    stk_drain(full0 + 8 * (uint32_t)(i % ST), (uint32_t)((i / ST) & 1));
}

// Activations for decode widths (BN <= 32), by the whole warp 2: lane 0 finds
// how many consecutive stages may be filled (weight box issued, inputs
// complete -- acquire loads of the producers' counters, no fences), then the
// 32 lanes copy up to NB stages' BN x 64 bf16 tiles from L2 into the ring in
// the 128-byte-swizzled layout the MMA descriptors expect, fence the shared
// writes for the tensor cores (async proxy) and arrive on each stage's full
// barrier (its second arrival; the weight box brings the transaction bytes).
template <int BN, int ST>
__device__ void stk_acts_ldg(const StackLaunch& L, uint8_t* smem, uint32_t full0, volatile int* abort_,
                             volatile long long* s_iw, volatile int* s_wdone) {
  using S = StkSmem<BN, ST>;
  const StackParams& P = L.P;
  const int lane = threadIdx.x & 31;
  constexpr int CPL = BN * 8 * kStkSub / 32;        // 16-byte chunks per lane per stage
  static_assert(CPL <= 16, "activation copy keeps at most 16 chunks per lane in flight");
  constexpr int NB = 16 / CPL;                      // stages per batch
  KbIter a;
  a.seek(P, 0);
  long long ia = 0;
  int sa = 0;
  // lane 0 only: inputs known complete below known_f in phase known_p
  int known_p = -1, known_f = 0;
  bool waited = false;
  unsigned long long idle_since = 0;
  uint32_t idles = 0;
  const int G = P.NH / P.NKV;
  auto kb_ready = [&](int f) -> bool { return unit_inputs_ready<true>(P, a, f, G); };
  for (;;) {
    int nb = 0, stop = 0;
    if (lane == 0) {
      if (!a.valid(P) || *abort_) {
        stop = 1;
      } else {
        if (!waited) {
          pdl_wait();
          waited = true;
        }
        if (known_p != a.p) {
          bool ok = true;
          bool per_kb = false;
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            const int k = a.dep_kind[i];
            if ((k == kDepTotLanes || k == kDepTotTiles) && ld_acquire_s32(P.tot + a.dep_off[i]) < a.dep_target[i])
              ok = false;
            per_kb |= k == kDepKbHead || k == kDepKbTile;
          }
          if (ok) {
            known_p = a.p;
            known_f = per_kb ? a.f : a.hi;
          }
        }
        if (known_p == a.p)
          while (known_f < a.hi && known_f < a.f + NB && kb_ready(known_f)) ++known_f;
        const long long iw = *s_iw;
        const long long lim = min(min((long long)NB, iw - ia), (long long)(a.hi - a.f));
        nb = known_p == a.p ? (int)min(lim, (long long)(known_f - a.f)) : 0;
        if (nb <= 0) {
          nb = 0;
          if (*s_wdone && ia >= *s_iw) {
            *abort_ = 1;   // weights stopped early
            stop = 1;
          } else if ((++idles & 63u) == 0) {
            const unsigned long long now = gtime_ns();
            if (idle_since == 0) idle_since = now;
            if (ld_volatile(P.err) != 0) {
              *abort_ = 1;
              stop = 1;
            } else if (now - idle_since > kStkWaitNs) {
              atomicExch(P.err, kDevTimeoutGrid);
              *abort_ = 1;
              stop = 1;
            }
          }
        } else {
          idle_since = 0;
          idles = 0;
          if (P.trace && a.f == a.lo) {
            stk_trace(P, a.p, 6);
            stk_trace(P, a.p, 3);
            stk_trace_value(P, a.p, 11, (unsigned long long)min((long long)(a.hi - a.f), iw - ia));
          }
        }
      }
    }
    stop = __shfl_sync(0xffffffffu, stop, 0);
    nb = __shfl_sync(0xffffffffu, nb, 0);
    if (stop) break;
    if (nb == 0) {
      __nanosleep(kStkPollNs);
      continue;
    }
    // copy nb stages (same phase): all loads first, then the stores
    const __nv_bfloat16* xb = P.x[a.xbuf];
    const long K = P.xK[a.xbuf];
    const int row0 = a.head ? 2 * P.head_lane0 : 0;
    const int rows = 2 * (a.head ? P.head_n : P.n);
    // chunk q of a stage: sub-tile q / (8 BN), row (q / 8) % BN, 16-byte chunk q % 8
    uint4 v[NB][CPL];
#pragma unroll
    for (int k = 0; k < NB; ++k) {
      const int kc = ((a.f + k) % a.KB) * kStkBK;
#pragma unroll
      for (int c = 0; c < CPL; ++c) {
        const int q = lane + 32 * c, u = q / (8 * BN), r = (q >> 3) % BN, j = q & 7;
        const int col = kc + u * kGemmBK + j * 8;
        v[k][c] = (k < nb && r < rows && col < K)
                      ? __ldcg(reinterpret_cast<const uint4*>(xb + (long)(row0 + r) * K + col))
                      : make_uint4(0u, 0u, 0u, 0u);
      }
    }
#pragma unroll
    for (int k = 0; k < NB; ++k) {
      if (k < nb) {
        int st = sa + k;
        if (st >= ST) st -= ST;
        uint8_t* tile = smem + st * S::kStage + S::kA;
#pragma unroll
        for (int c = 0; c < CPL; ++c) {
          const int q = lane + 32 * c, u = q / (8 * BN), r = (q >> 3) % BN, j = q & 7;
          *reinterpret_cast<uint4*>(tile + u * S::kSubB + r * 128 + ((j ^ (r & 7)) << 4)) = v[k][c];
        }
        fence_proxy_async();   // shared writes -> tensor-core (async proxy) reads
        __syncwarp();
        if (lane == 0) mbar_arrive(full0 + 8 * (uint32_t)st);
      }
    }
    if (lane == 0 && P.trace && a.f + nb == a.hi) stk_trace(P, a.p, 8);
    for (int k = 0; k < nb; ++k) a.step(P);
    ia += nb;
    sa += nb;
    if (sa >= ST) sa -= ST;
  }
  // Exit. Normally every stage has been filled. When aborting, arrive on the
  // stages whose weight box was issued (their tiles are discarded) so their
  // barriers complete, then wait until all boxes have landed.
  if (lane == 0) {
    const unsigned long long t0 = gtime_ns();
    while (!*s_wdone && gtime_ns() - t0 < kStkWaitNs) __nanosleep(64);
    const long long iw = *s_iw;
    for (long long i = ia; i < iw; ++i) {
      mbar_arrive(full0 + 8 * (uint32_t)sa);
      if (++sa == ST) sa = 0;
    }
    if (ia < iw && ld_volatile(P.err) == 0) atomicExch(P.err, kDevTimeoutGrid);
    for (long long i = iw > ST ? iw - ST : 0; i < iw; ++i)
      stk_drain(full0 + 8 * (uint32_t)(i % ST), (uint32_t)((i / ST) & 1));
  }
}

// ------------------------------------------------------------- MMA issuer
// Segment j accumulates into TMEM columns [(j & 1) * BN, +BN); before reusing
// a buffer it waits until the epilogue warps have read segment j - 2.
template <int BN, int ST>
__device__ void stk_mma(const StackParams& P, uint8_t* smem, uint32_t full0, uint32_t empty0,
                        uint32_t accf0, uint32_t acce0, uint32_t fin, uint32_t tmem, volatile int* abort_) {
  // (reads only the program: phases and KbIter)
  using S = StkSmem<BN, ST>;
  constexpr uint32_t idesc = umma_idesc_bf16(kGemmBM, BN);
  KbIter m;
  m.seek(P, 0);
  long i = 0;
  int seg = 0;
  int ms = 0;          // ring stage of k-block i
  uint32_t mpar = 0;   // its fill parity
  while (m.valid(P) && !*abort_) {
    const int p0 = m.p;
    const int t = m.f / m.KB;
    const int send = min(m.hi, (t + 1) * m.KB);
    const int seg_lo = m.lo, seg_hi = m.hi, seg_kb = m.KB;
    const int b = seg & 1;
    if (seg >= 2 && !stk_wait(acce0 + 8 * b, (uint32_t)(((seg >> 1) - 1) & 1), abort_, P.err, kDevTimeoutAcc))
      break;
    tc_fence_after();
    const uint32_t d = tmem + (uint32_t)(b * BN);
    bool first = true, ok = true;
    do {
      const int s = ms;
      if (!stk_wait(full0 + 8 * s, mpar, abort_, P.err, kDevTimeoutFull)) {
        ok = false;
        break;
      }
      tc_fence_after();
      stk_log(P, 2, i);
      if (P.trace && first && m.f == seg_lo) stk_trace(P, p0, 9);
      const uint32_t a_s = smem_u32(smem + s * S::kStage);
      const uint32_t b_s = a_s + S::kA;
#pragma unroll
      for (int u = 0; u < kStkSub; ++u)
#pragma unroll
        for (int k = 0; k < kGemmBK / 16; ++k)
          tc_mma_bf16(d, umma_desc_sw128(a_s + u * S::kSubA + 32 * k),
                      umma_desc_sw128(b_s + u * S::kSubB + 32 * k), idesc, (first && u == 0 && k == 0) ? 0u : 1u);
      first = false;
      stk_log(P, 1, i);
      tc_commit(empty0 + 8 * s);
      stk_log(P, 3, i);
      ++i;
      if (++ms == ST) {
        ms = 0;
        mpar ^= 1u;
      }
      m.step(P);
    } while (m.valid(P) && m.p == p0 && m.f < send);
    if (!ok) break;
    tc_commit(accf0 + 8 * b);
    if (P.trace && send == min(seg_hi, (seg_lo / seg_kb + 1) * seg_kb)) stk_trace(P, p0, 10);
    ++seg;
  }
  // every MMA this thread issued completes before the TMEM is released
  if (i > 0) {
    tc_commit(fin);
    stk_drain(fin, 0);
  }
}

// ---------------------------------------------------------- GEMM epilogue
// Partial slot of CTA c for tile t: 0 if t is the CTA's first segment, else 1;
// two sets, by the parity of the GEMM phase (a GEMM phase transitively waits
// for every tile of the GEMM phase two before it, never for the one before).
__device__ __forceinline__ float* seg_slot(const StackParams& P, int BNh, int par, int c, int slot) {
  return P.part_ws + (long)((par * (int)gridDim.x + c) * 2 + slot) * BNh * kGemmBM;
}

// Sum tile t's partials over its contributors in CTA order and apply the
// phase's epilogue. 128 epilogue threads; a unit is a pair of rows that one
// epilogue needs together (RoPE pair, gate/up pair, or two adjacent rows).
template <int BN>
__device__ void stk_gemm_finish(const StackParams& P, const Phase& ph, int t, int2 cc, const KRange& rg,
                                int lanes) {
  const int et = threadIdx.x - kStkEpiTid0;
  const int m0 = t * kGemmBM;
  for (int item = et; item < 64 * lanes; item += 128) {
    const int l = item >> 6, u = item & 63;
    int r0, r1;
    if (ph.epi == kEpiQkvRope) {
      const int half = P.HD / 2;
      r0 = (u / half) * P.HD + (u % half);
      r1 = r0 + half;
    } else if (ph.epi == kEpiSwiGLU) {
      r0 = u;
      r1 = u + kGemmBM / 2;
    } else {
      r0 = 2 * u;
      r1 = 2 * u + 1;
    }
    // all loads of a batch of 8 contributors first, then the adds in CTA order
    float v0 = 0.f, v1 = 0.f;
    for (int c0 = cc.x; c0 <= cc.y; c0 += 8) {
      float a0[8], a1[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int c = c0 + j;
        a0[j] = 0.f;
        a1[j] = 0.f;
        if (c <= cc.y) {
          const int lo_c = (int)((long)c * rg.T / rg.Gw);
          const float* pp = seg_slot(P, BN / 2, ph.gemm_idx & 1, c, lo_c >= t * ph.KB ? 0 : 1) + l * kGemmBM;
          a0[j] = __ldcg(pp + r0);
          a1[j] = __ldcg(pp + r1);
        }
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        v0 += a0[j];
        v1 += a1[j];
      }
    }
    if (ph.epi == kEpiStore) {
      if (m0 + r0 < ph.Mw) ph.out[(long)l * ph.Mw + m0 + r0] = v0;
      if (m0 + r1 < ph.Mw) ph.out[(long)l * ph.Mw + m0 + r1] = v1;
    } else if (ph.epi == kEpiSwiGLU) {
      const int i = t * (kGemmBM / 2) + u;
      if (i < P.I) store_pair(P.x[kXAct], P.I, l, i, v0 / (1.f + expf(-v0)) * v1);
    } else {
      const int hd = P.HD, half = hd / 2;
      const int mg = m0 + r0;
      const int head = mg / hd, i = mg - head * hd;   // i < half
      const int pos = P.meta.get(kMetaPos, l);
      const int slot = P.meta.get(kMetaSlot, l);
      const int kvd = P.NKV * hd;
      const bool slot_ok = slot >= 0 && slot < P.n_slots;
      if (head < P.NH + P.NKV) {
        float sn, cs;
        sincosf((float)pos * P.inv_freq[i], &sn, &cs);
        const float y0 = v0 * cs - v1 * sn, y1 = v1 * cs + v0 * sn;
        if (head < P.NH) {
          float* qr = P.q + (long)l * P.NH * hd + head * hd;
          qr[i] = y0;
          qr[i + half] = y1;
        } else if (slot_ok) {
          __nv_bfloat16* kr = ph.kpool + (long)slot * kvd + (head - P.NH) * hd;
          kr[i] = f2bf(y0);
          kr[i + half] = f2bf(y1);
        } else {
          atomicExch(P.err, kDevBadIndex);
        }
      } else if (slot_ok) {
        __nv_bfloat16* vr = ph.vpool + (long)slot * kvd + (head - P.NH - P.NKV) * hd;
        vr[i] = f2bf(v0);
        vr[i + half] = f2bf(v1);
      }
    }
  }
}

// The epilogue warps' part of a GEMM phase: for each of this CTA's segments,
// read the accumulator (hi + lo column of each lane), publish the partial,
// release the accumulator, and finish the tile if this CTA is its last
// contributor. Returns false if the CTA is aborting (uniform over the 128
// threads: the single waiting thread broadcasts its result).
template <int BN>
__device__ bool stk_gemm_epilogue(const StackParams& P, const Phase& ph, int phase, int& seg, uint32_t accf0,
                                  uint32_t acce0, uint32_t tmem, volatile int* abort_, int* s_flag) {
  const KRange rg = gemm_range(ph);
  const int et = threadIdx.x - kStkEpiTid0;
  const int q = (threadIdx.x >> 5) & 3;             // TMEM lane quadrant of this warp
  const int r = q * 32 + (threadIdx.x & 31);        // tile row read by this thread
  const int lanes = ph.head ? P.head_n : P.n;
  for (int f = rg.lo; f < rg.hi;) {
    const int t = f / ph.KB;
    const int send = min(rg.hi, (t + 1) * ph.KB);
    const int b = seg & 1;
    if (et == 0) {
      s_flag[0] = stk_wait(accf0 + 8 * b, (uint32_t)((seg >> 1) & 1), abort_, P.err, kDevTimeoutAcc);
      if (P.trace && f == rg.lo) stk_trace(P, phase, 2);
    }
    named_bar(kBarEpi, 128);
    if (!s_flag[0]) return false;
    tc_fence_after();
    float* mine = seg_slot(P, BN / 2, ph.gemm_idx & 1, blockIdx.x, rg.lo >= t * ph.KB ? 0 : 1);
    const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * BN);
#pragma unroll 1
    for (int c0 = 0; c0 < 2 * lanes; c0 += 8) {
      uint32_t v[8];
      tmem_ld_32x32b_x8(taddr + (uint32_t)c0, v);
      tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int l = c0 / 2 + j;
        if (l < lanes) mine[l * kGemmBM + r] = __uint_as_float(v[2 * j]) + __uint_as_float(v[2 * j + 1]);
      }
    }
    tc_fence_before();
    mbar_arrive(acce0 + 8 * b);
    named_bar(kBarEpi, 128);
    const int2 cc = tile_ctas(t, ph.KB, rg.T, rg.Gw);
    bool last = true;
    if (cc.x != cc.y) {
      // the ticket releases this CTA's partial (written by the 128 threads
      // before the barrier) and acquires the others' for the last one
      if (et == 0) {
        int* tk = P.tile_tickets + (ph.gemm_idx & 1) * P.ticket_stride + t;
        const int ticket = atom_acq_rel_add(tk, 1);
        s_flag[1] = ticket == cc.y - cc.x;
        if (s_flag[1]) *tk = 0;   // all contributors arrived: ready for the next use
      }
      named_bar(kBarEpi, 128);
      last = s_flag[1] != 0;
    }
    if (last) {
      stk_gemm_finish<BN>(P, ph, t, cc, rg, lanes);
      publish(kBarEpi, 128, et == 0, P.cnt + ph.cnt_off + t, P.tot + phase, !ActPath<BN>::kLdg);   // tile t stored
    }
    named_bar(kBarEpi, 128);   // slot and flags free for the next segment
    ++seg;
    f = send;
  }
  if (et == 0) stk_trace(P, phase, 7);
  return true;
}

// --------------------------------------------------------------- attention
// Work item = (lane, kv head, chunk of kStkChunk positions), numbered over the
// lanes' actual chunk counts and dealt to CTAs round-robin. Each sub-group of
// HD/8 threads owns PER fixed positions of the chunk; the chunk's slot ids and
// the query load together, then every K and V row of the sub-group is loaded
// at once (16 bytes per thread per row), so an item costs two dependent memory
// round trips before its partial (acc, max, sum) is written. The last item of
// a (lane, kv head) to finish (ticket) merges the chunks in chunk order, eight
// at a time with a running max, and writes the O projection's (hi, lo) input.
// Chunk boundaries are fixed multiples of kStkChunk and positions map to
// sub-groups by index, so results do not depend on the batch.
// Inputs of the attention items of kv head g: the QKV tiles holding g's q, k
// and v rows (or the QK-norm phase), and the timeline mapping update.
__device__ __forceinline__ bool wait_attn_inputs(const StackParams& P, const Phase& ph, int g,
                                                 volatile int* abort_) {
  const int G = P.NH / P.NKV, HD = P.HD, QD = P.NH * HD, KVD = P.NKV * HD;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int k = ph.dep_kind[i], q = ph.dep_phase[i];
    if (k == kDepQkvHead) {
      const int* c = P.cnt + P.phases[q].cnt_off;
      const int ranges[3][2] = {{g * G * HD, (g + 1) * G * HD},
                                {QD + g * HD, QD + (g + 1) * HD},
                                {QD + KVD + g * HD, QD + KVD + (g + 1) * HD}};
      for (int r = 0; r < 3; ++r)
        for (int t = ranges[r][0] / kGemmBM; t <= (ranges[r][1] - 1) / kGemmBM; ++t)
          if (!grid_wait(reinterpret_cast<const unsigned*>(c + t), 1u, abort_, P.err, kDevTimeoutGrid,
                         kStkWaitNs))
            return false;
    } else if (k == kDepTotLanes || k == kDepTotTiles) {
      if (!grid_wait(reinterpret_cast<const unsigned*>(P.tot + q), (unsigned)dep_tot_target(P, k, q), abort_,
                     P.err, kDevTimeoutGrid, kStkWaitNs))
        return false;
    }
  }
  return true;
}

template <int HD>
__device__ bool stk_attention(const StackParams& P, const Phase& ph, int phase, uint8_t* work,
                              volatile int* abort_, int* s_flag, bool proxy) {
  constexpr int GM = HD == 128 ? 2 : 4;      // query heads per KV head supported
  constexpr int LPP = HD / 8;
  constexpr int PPW = 32 / LPP;
  constexpr int NW = kStkWorkers / 32;
  constexpr int NSG = NW * PPW;
  constexpr int PER = kStkChunk / NSG;
  static_assert(PER * NSG == kStkChunk, "chunk must split evenly over sub-groups");
  int* s_pref = reinterpret_cast<int*>(work);                  // [lanes + 1]
  int* s_slot = s_pref + kStkMaxLanes + 4;                     // [kStkChunk]
  float* sm_m = reinterpret_cast<float*>(s_slot + kStkChunk);  // [NW][GM]
  float* sm_l = sm_m + NW * GM;
  float* sm_acc = sm_l + NW * GM;                              // [NW][GM][HD]
  int* s_last = reinterpret_cast<int*>(sm_acc + NW * GM * HD);

  const int wt = threadIdx.x - kStkWorkerTid0;
  const int warp = wt >> 5, lane = threadIdx.x & 31;
  const int sub = lane / LPP, sl = lane % LPP;
  const int sg = warp * PPW + sub;
  const int G = P.NH / P.NKV;
  const int kd = P.NKV * HD;
  // items per lane (parallel), then an exclusive scan by the first warp
  for (int b = wt; b < P.n; b += kStkWorkers) {
    const int T = P.meta.get(kMetaPos, b) + 1;
    const bool ok = T >= 1 && T <= P.max_ctx;
    if (!ok) atomicExch(P.err, kDevBadIndex);
    s_pref[b + 1] = ok ? P.NKV * ((T + kStkChunk - 1) / kStkChunk) : 0;
  }
  named_bar(kBarWorkers, kStkWorkers);
  if (warp == 0) {
    int carry = 0;
    for (int base = 0; base < P.n; base += 32) {
      const int b = base + lane;
      int x = b < P.n ? s_pref[b + 1] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
      }
      if (b < P.n) s_pref[b + 1] = carry + x;
      carry += __shfl_sync(0xffffffffu, x, 31);
    }
    if (lane == 0) s_pref[0] = 0;
  }
  named_bar(kBarWorkers, kStkWorkers);
  const int total = s_pref[P.n];
  for (int it = blockIdx.x; it < total; it += gridDim.x) {
    int b = 0;
    while (s_pref[b + 1] <= it) ++b;
    const int nch = (s_pref[b + 1] - s_pref[b]) / P.NKV;
    const int rem = it - s_pref[b];
    const int g = rem / nch, c = rem - g * nch;
    if (wt == 0) s_flag[2] = wait_attn_inputs(P, ph, g, abort_);
    named_bar(kBarWorkers, kStkWorkers);
    if (!s_flag[2]) return false;
    const bool first_item = it == (int)blockIdx.x;
    if (wt == 0 && first_item) stk_trace(P, phase, 2);   // inputs complete
    const int T = P.meta.get(kMetaPos, b) + 1;
    const int row = P.meta.get(kMetaRow, b);
    const bool row_ok = row >= 0 && row < P.rows;
    const int start = c * kStkChunk;
    const int n_in = min(kStkChunk, T - start);
    const int* mrow = P.map + (long)(row_ok ? row : 0) * P.max_ctx + start;
    // slot ids of the chunk and this thread's query slice, loaded together
    int sv = -1;
    if (wt < kStkChunk && row_ok && wt < n_in) sv = __ldcg(mrow + wt);
    float qv[GM][8];
#pragma unroll
    for (int h = 0; h < GM; ++h) {
#pragma unroll
      for (int d = 0; d < 8; ++d) qv[h][d] = 0.f;
      if (h < G) {
        const float* qp = P.q + (long)b * P.NH * HD + (g * G + h) * HD + sl * 8;
        const float4 q0 = ldcg4(qp), q1 = ldcg4(qp + 4);
        const float qq[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
        for (int d = 0; d < 8; ++d) qv[h][d] = qq[d] * P.attn_scale;
      }
    }
    if (wt < kStkChunk) {
      if (sv >= P.n_slots || (sv < 0 && row_ok && wt < n_in)) {
        atomicExch(P.err, kDevBadIndex);
        sv = -1;
      }
      s_slot[wt] = sv;
    }
    if (!row_ok && wt == 0) atomicExch(P.err, kDevBadIndex);
    named_bar(kBarWorkers, kStkWorkers);

    uint4 kr[PER], vr[PER];
#pragma unroll
    for (int t = 0; t < PER; ++t) {
      const int slot = s_slot[sg + t * NSG];
      const long off = (long)slot * kd + g * HD + sl * 8;
      kr[t] = slot >= 0 ? __ldcg(reinterpret_cast<const uint4*>(ph.kpool + off)) : make_uint4(0, 0, 0, 0);
      vr[t] = slot >= 0 ? __ldcg(reinterpret_cast<const uint4*>(ph.vpool + off)) : make_uint4(0, 0, 0, 0);
    }
    float sc[GM][PER];
#pragma unroll
    for (int t = 0; t < PER; ++t) {
      float kf[8];
      unpack8(kr[t], kf);
#pragma unroll
      for (int h = 0; h < GM; ++h) {
        float s = 0.f;
#pragma unroll
        for (int d = 0; d < 8; ++d) s += qv[h][d] * kf[d];
#pragma unroll
        for (int o = LPP / 2; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        sc[h][t] = s_slot[sg + t * NSG] >= 0 ? s : -INFINITY;
      }
    }
    float m[GM], l[GM], acc[GM][8];
#pragma unroll
    for (int h = 0; h < GM; ++h) {
      m[h] = -INFINITY;
#pragma unroll
      for (int t = 0; t < PER; ++t) m[h] = fmaxf(m[h], sc[h][t]);
      l[h] = 0.f;
#pragma unroll
      for (int d = 0; d < 8; ++d) acc[h][d] = 0.f;
    }
#pragma unroll
    for (int t = 0; t < PER; ++t) {
      float vf[8];
      unpack8(vr[t], vf);
#pragma unroll
      for (int h = 0; h < GM; ++h) {
        const float p = m[h] == -INFINITY ? 0.f : __expf(sc[h][t] - m[h]);
        l[h] += p;
#pragma unroll
        for (int d = 0; d < 8; ++d) acc[h][d] += p * vf[d];
      }
    }
#pragma unroll
    for (int h = 0; h < GM; ++h) {
#pragma unroll
      for (int o = LPP; o < 32; o <<= 1) {
        const float m2 = __shfl_xor_sync(0xffffffffu, m[h], o);
        const float l2 = __shfl_xor_sync(0xffffffffu, l[h], o);
        const float mn = fmaxf(m[h], m2);
        const float c1 = mn == -INFINITY ? 0.f : __expf(m[h] - mn);
        const float c2 = mn == -INFINITY ? 0.f : __expf(m2 - mn);
        l[h] = l[h] * c1 + l2 * c2;
#pragma unroll
        for (int d = 0; d < 8; ++d) {
          const float a2 = __shfl_xor_sync(0xffffffffu, acc[h][d], o);
          acc[h][d] = acc[h][d] * c1 + a2 * c2;
        }
        m[h] = mn;
      }
      if (sub == 0) {
#pragma unroll
        for (int d = 0; d < 8; ++d) sm_acc[(warp * GM + h) * HD + sl * 8 + d] = acc[h][d];
        if (sl == 0) {
          sm_m[warp * GM + h] = m[h];
          sm_l[warp * GM + h] = l[h];
        }
      }
    }
    named_bar(kBarWorkers, kStkWorkers);
    if (wt == 0 && first_item) stk_trace(P, phase, 4);   // scores and values done
    for (int t = wt; t < G * HD; t += kStkWorkers) {
      const int h = t / HD, d = t - h * HD;
      float mm = -INFINITY;
#pragma unroll
      for (int w = 0; w < NW; ++w) mm = fmaxf(mm, sm_m[w * GM + h]);
      float ll = 0.f, aa = 0.f;
#pragma unroll
      for (int w = 0; w < NW; ++w) {
        const float cw = mm == -INFINITY ? 0.f : __expf(sm_m[w * GM + h] - mm);
        ll += sm_l[w * GM + h] * cw;
        aa += sm_acc[(w * GM + h) * HD + d] * cw;
      }
      const long idx = ((long)b * P.NH + g * G + h) * P.max_chunks + c;
      P.o_part[idx * HD + d] = aa;
      if (d == 0) {
        P.ml_part[idx * 2] = mm;
        P.ml_part[idx * 2 + 1] = ll;
      }
    }
    named_bar(kBarWorkers, kStkWorkers);
    if (wt == 0) {
      int* tk = P.attn_tickets + (long)b * P.NKV + g;
      const int ticket = atom_acq_rel_add(tk, 1);   // releases this chunk, acquires the others
      s_last[0] = ticket == nch - 1;
      if (s_last[0]) *tk = 0;
    }
    named_bar(kBarWorkers, kStkWorkers);
    if (wt == 0 && first_item) stk_trace(P, phase, 5);   // ticket taken
    if (s_last[0]) {
      for (int t = wt; t < G * HD; t += kStkWorkers) {
        const int h = t / HD, d = t - h * HD;
        const long base = ((long)b * P.NH + g * G + h) * P.max_chunks;
        // chunks in order, eight loads in flight at a time, running max
        float mm = -INFINITY, ll = 0.f, aa = 0.f;
        for (int c0 = 0; c0 < nch; c0 += 8) {
          float cm[8], cl[8], co[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            cm[j] = -INFINITY;
            cl[j] = 0.f;
            co[j] = 0.f;
            if (c0 + j < nch) {
              const float2 ml = __ldcg(reinterpret_cast<const float2*>(P.ml_part + (base + c0 + j) * 2));
              cm[j] = ml.x;
              cl[j] = ml.y;
              co[j] = __ldcg(P.o_part + (base + c0 + j) * HD + d);
            }
          }
          float bm = mm;
#pragma unroll
          for (int j = 0; j < 8; ++j) bm = fmaxf(bm, cm[j]);
          const float r = bm == -INFINITY ? 0.f : __expf(mm - bm);
          ll *= r;
          aa *= r;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float w = bm == -INFINITY ? 0.f : __expf(cm[j] - bm);
            ll += cl[j] * w;
            aa += co[j] * w;
          }
          mm = bm;
        }
        store_pair(P.x[kXAttn], (long)P.NH * HD, b, (g * G + h) * HD + d, ll > 0.f ? aa / ll : 0.f);
      }
      publish(kBarWorkers, kStkWorkers, wt == 0, P.cnt + ph.cnt_off + g, P.tot + phase, proxy);   // (b, g) merged
    }
    named_bar(kBarWorkers, kStkWorkers);   // shared scratch free for the next item
  }
  return true;
}

// ------------------------------------------------------------ per-lane rows
// Per-lane phases run one lane per call (lanes dealt to CTAs round-robin),
// 192 threads, each thread holding NV float4 columns. With NV = 3 (H <= 2304, every preset)
// all of a row's loads -- inputs, residual and the bf16 norm weights -- are
// issued before the first use, so a row costs one memory round trip plus its
// block reductions; larger rows (NV = 8) load the weights at use.
__device__ __forceinline__ uint2 ldg_u2(const __nv_bfloat16* p) {
  return __ldg(reinterpret_cast<const uint2*>(p));
}

__device__ __forceinline__ float4 bf4_of(uint2 u) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
  const float2 a = __bfloat1622float2(h[0]), b = __bfloat1622float2(h[1]);
  return make_float4(a.x, a.y, b.x, b.y);
}

constexpr uint2 kBf16Ones = {0x3F803F80u, 0x3F803F80u};   // four bf16 1.0

template <int NV>
__device__ __forceinline__ void stk_store_row(const StackParams& P, const Phase& ph, int b, float4* v,
                                              float ss, float* red, const uint2* wx) {
  const int wt = threadIdx.x - kStkWorkerTid0;
  const int H = P.H, H4 = H / 4;
  float inv = 1.f;
  const bool wxo = ph.x_out >= 0;
  if (wxo && ph.x_norm_w) inv = rsqrtf(worker_sum(ss, red) / H + P.eps);
  int so = -1;
  if (ph.bank) {
    so = P.meta.get(kMetaStateOut, b);
    if (so < 0 || so >= P.bank_rows) {
      if (wt == 0) atomicExch(P.err, kDevBadIndex);
      so = -1;
    }
  }
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int j = wt + k * kStkWorkers;
    if (j >= H4) continue;
    if (ph.out_h) *reinterpret_cast<float4*>(ph.out_h + (long)b * H + 4 * j) = v[k];
    if (so >= 0) *reinterpret_cast<float4*>(ph.bank + (long)so * H + 4 * j) = v[k];
    if (wxo) {
      float4 x = v[k];
      if (ph.x_norm_w) x = f4_scale(v[k], inv, wx ? bf4_of(wx[k]) : ld_bf4(ph.x_norm_w + 4 * j));
      store_pair4(P.x[ph.x_out], P.xK[ph.x_out], b, 4 * j, x);
    }
  }
}

// a = src[b] (+ bias); a = a_norm ? rms(a) * wa : a; out = resid + a;
// out = final_norm ? rms(out) * wf : out; then out_h / bank / x as in
// resid_epi_kernel.
template <int NV, bool UPFRONT>
__device__ void stk_row_impl(const StackParams& P, const Phase& ph, int b, float* red, int tp) {
  const int wt = threadIdx.x - kStkWorkerTid0;
  const int H = P.H, H4 = H / 4;
  const bool tr = P.trace && wt == 0 && blockIdx.x == 0 && b == 0;
  const long long c0 = clock64();
  float4 v[NV], rr[NV];
  uint2 wa[UPFRONT ? NV : 1], wf[UPFRONT ? NV : 1], wx[UPFRONT ? NV : 1], bi[UPFRONT ? NV : 1];
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int j = wt + k * kStkWorkers;
    const bool on = j < H4;
    v[k] = on ? ldcg4(ph.src + (long)b * H + 4 * j) : make_float4(0.f, 0.f, 0.f, 0.f);
    rr[k] = on && ph.resid ? ldcg4(ph.resid + (long)b * H + 4 * j) : make_float4(0.f, 0.f, 0.f, 0.f);
    if (UPFRONT) {
      wa[k] = on && ph.a_norm_w ? ldg_u2(ph.a_norm_w + 4 * j) : kBf16Ones;
      wf[k] = on && ph.final_norm_w ? ldg_u2(ph.final_norm_w + 4 * j) : kBf16Ones;
      wx[k] = on && ph.x_norm_w ? ldg_u2(ph.x_norm_w + 4 * j) : kBf16Ones;
      bi[k] = on && ph.bias ? ldg_u2(ph.bias + 4 * j) : make_uint2(0u, 0u);
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int j = wt + k * kStkWorkers;
    if (ph.bias && j < H4) v[k] = f4_add(v[k], UPFRONT ? bf4_of(bi[k]) : ld_bf4(ph.bias + 4 * j));
    ss += f4_sq(v[k]);
  }
  if (ph.a_norm_w) {
    const float inv = rsqrtf(worker_sum(ss, red) / H + P.eps);
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int j = wt + k * kStkWorkers;
      if (j < H4) v[k] = f4_scale(v[k], inv, UPFRONT ? bf4_of(wa[k]) : ld_bf4(ph.a_norm_w + 4 * j));
    }
  }
  ss = 0.f;
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    v[k] = f4_add(v[k], rr[k]);
    ss += f4_sq(v[k]);
  }
  if (ph.final_norm_w) {
    const float inv = rsqrtf(worker_sum(ss, red) / H + P.eps);
    ss = 0.f;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int j = wt + k * kStkWorkers;
      if (j < H4) v[k] = f4_scale(v[k], inv, UPFRONT ? bf4_of(wf[k]) : ld_bf4(ph.final_norm_w + 4 * j));
      ss += f4_sq(v[k]);
    }
  }
  if (tr) stk_trace_value(P, tp, 8, (unsigned long long)(clock64() - c0));   // before the stores
  stk_store_row<NV>(P, ph, b, v, ss, red, UPFRONT ? wx : nullptr);
  if (tr) stk_trace_value(P, tp, 9, (unsigned long long)(clock64() - c0));   // stores issued
}

__device__ void stk_row(const StackParams& P, const Phase& ph, int b, float* red, int tp) {
  if (P.H <= 4 * 3 * kStkWorkers) stk_row_impl<3, true>(P, ph, b, red, tp);
  else stk_row_impl<kStkRowNV, false>(P, ph, b, red, tp);
}

// h = embedding(token) * scale (src null) or src[state_in]; then out_h /
// bank / x (prep_kernel semantics).
template <int NV, bool UPFRONT>
__device__ void stk_prep_impl(const StackParams& P, const Phase& ph, int b, float* red) {
  const int wt = threadIdx.x - kStkWorkerTid0;
  const int H = P.H, H4 = H / 4;
  int src;
  if (!ph.src) {
    src = P.meta.get(kMetaToken, b);
    if (src < 0 || src >= P.vocab) src = -1;
  } else {
    src = P.meta.get(kMetaStateIn, b);
    if (src < 0 || src >= P.bank_rows) src = -1;
  }
  if (src < 0 && wt == 0) atomicExch(P.err, kDevBadIndex);
  float4 v[NV];
  uint2 wx[UPFRONT ? NV : 1];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int j = wt + k * kStkWorkers;
    v[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (j < H4 && src >= 0) {
      if (!ph.src) {
        const float4 e = ld_bf4(P.embed + (long)src * H + 4 * j);
        v[k] = make_float4(e.x * P.embed_scale, e.y * P.embed_scale, e.z * P.embed_scale,
                           e.w * P.embed_scale);
      } else {
        v[k] = ldcg4(ph.src + (long)src * H + 4 * j);
      }
    }
    if (UPFRONT) wx[k] = j < H4 && ph.x_norm_w ? ldg_u2(ph.x_norm_w + 4 * j) : kBf16Ones;
    ss += f4_sq(v[k]);
  }
  stk_store_row<NV>(P, ph, b, v, ss, red, UPFRONT ? wx : nullptr);
}

__device__ void stk_prep(const StackParams& P, const Phase& ph, int b, float* red) {
  if (P.H <= 4 * 3 * kStkWorkers) stk_prep_impl<3, true>(P, ph, b, red);
  else stk_prep_impl<kStkRowNV, false>(P, ph, b, red);
}

// Raven adapter input: x_cat[b] = (hi, lo) of [bank_h[state_in], bank_inj[state_in]].
__device__ void stk_cat(const StackParams& P, int b) {
  const int wt = threadIdx.x - kStkWorkerTid0;
  const int H = P.H;
  const int si = P.meta.get(kMetaStateIn, b);
  if (si < 0 || si >= P.bank_rows) {
    if (wt == 0) atomicExch(P.err, kDevBadIndex);
    return;
  }
  for (int j = wt; j < H / 4; j += kStkWorkers) {
    store_pair4(P.x[kXCat], 2L * H, b, 4 * j, ldcg4(P.bank_h + (long)si * H + 4 * j));
    store_pair4(P.x[kXCat], 2L * H, b, H + 4 * j, ldcg4(P.bank_inj + (long)si * H + 4 * j));
  }
}

// Timeline mapping (map_update_kernel): fork copy, then row[pos] = slot.
__device__ void stk_map(const StackParams& P, int b) {
  const int wt = threadIdx.x - kStkWorkerTid0;
  const int row = P.meta.get(kMetaRow, b), pos = P.meta.get(kMetaPos, b);
  const int frow = P.meta.get(kMetaForkRow, b), flen = P.meta.get(kMetaForkLen, b);
  if (row < 0 || row >= P.rows || pos < 0 || pos >= P.max_ctx ||
      (frow >= 0 && (frow >= P.rows || flen > P.max_ctx))) {
    if (wt == 0) atomicExch(P.err, kDevBadIndex);
    return;
  }
  int* dst = P.map + (long)row * P.max_ctx;
  if (frow >= 0) {
    const int* src = P.map + (long)frow * P.max_ctx;
    for (int j = wt; j < flen; j += kStkWorkers) dst[j] = __ldcg(src + j);
  }
  if (wt == 0) dst[pos] = P.meta.get(kMetaSlot, b);
}

// OLMo2 QK-norm over the stored QKV row of each lane (src [lanes][D]), neox
// RoPE, K/V written to the layer's pools, q kept in fp32 (qkv_epi_kernel).
__device__ void stk_qknorm(const StackParams& P, const Phase& ph, int b, float* red) {
  const int wt = threadIdx.x - kStkWorkerTid0;
  const int hd = P.HD, half = hd / 2;
  const int qd = P.NH * hd, kd = P.NKV * hd, D = qd + 2 * kd;
  const float* row = ph.src + (long)b * D;
  float ssq = 0.f, ssk = 0.f;
  for (int i = wt; i < qd + kd; i += kStkWorkers) {
    const float v = __ldcg(row + i);
    if (i < qd) ssq += v * v;
    else ssk += v * v;
  }
  const float iq = rsqrtf(worker_sum(ssq, red) / qd + P.eps);
  const float ik = rsqrtf(worker_sum(ssk, red) / kd + P.eps);
  const int pos = P.meta.get(kMetaPos, b);
  const int slot = P.meta.get(kMetaSlot, b);
  const bool slot_ok = slot >= 0 && slot < P.n_slots;
  if (!slot_ok && wt == 0) atomicExch(P.err, kDevBadIndex);
  const int pairs = (P.NH + P.NKV) * half;
  for (int t = wt; t < pairs; t += kStkWorkers) {
    const int head = t / half, i = t - head * half;
    const int base = head * hd;
    const bool isq = head < P.NH;
    const float sc = isq ? iq : ik;
    const __nv_bfloat16* nw = isq ? ph.q_norm_w + base : ph.k_norm_w + (base - qd);
    const float x1 = __ldcg(row + base + i) * sc * bf2f(nw[i]);
    const float x2 = __ldcg(row + base + i + half) * sc * bf2f(nw[i + half]);
    float sn, cs;
    sincosf((float)pos * P.inv_freq[i], &sn, &cs);
    const float y1 = x1 * cs - x2 * sn, y2 = x2 * cs + x1 * sn;
    if (isq) {
      P.q[(long)b * qd + base + i] = y1;
      P.q[(long)b * qd + base + i + half] = y2;
    } else if (slot_ok) {
      __nv_bfloat16* kr = ph.kpool + (long)slot * kd + (base - qd);
      kr[i] = f2bf(y1);
      kr[i + half] = f2bf(y2);
    }
  }
  if (slot_ok)
    for (int i = wt; i < kd; i += kStkWorkers)
      ph.vpool[(long)slot * kd + i] = f2bf(__ldcg(row + qd + kd + i));
}

// Raven hidden init (raven_init_kernel): bank_h[state_out] = position-keyed
// truncated normal; bank_inj[state_out] = h[b].
__device__ void stk_raven_init(const StackParams& P, int b) {
  const int wt = threadIdx.x - kStkWorkerTid0;
  const int H = P.H;
  const int so = P.meta.get(kMetaStateOut, b);
  if (so < 0 || so >= P.bank_rows) {
    if (wt == 0) atomicExch(P.err, kDevBadIndex);
    return;
  }
  const uint32_t pos = (uint32_t)P.meta.get(kMetaPos, b);
  const double lo = 0.0013498980316300946;  // Phi(-3)
  for (int i4 = wt; i4 < (H + 3) / 4; i4 += kStkWorkers) {
    const uint4 w = philox4x32_10(make_uint4((uint32_t)i4, pos, 0u, 0u), (uint32_t)P.init_seed,
                                  (uint32_t)(P.init_seed >> 32));
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int i = i4 * 4 + k;
      if (i >= H) break;
      const double u = ((double)(ws[k] >> 8) + 0.5) / 16777216.0;
      const double p = lo + u * (1.0 - 2.0 * lo);
      const double x = 1.4142135623730951 * erfinv(2.0 * p - 1.0);
      P.bank_h[(long)so * H + i] = P.init_std > 0.f ? (float)(x * P.init_std * P.embed_scale) : 0.f;
    }
  }
  for (int i = wt; i < H; i += kStkWorkers) P.bank_inj[(long)so * H + i] = __ldcg(P.h + (long)b * H + i);
}

// ------------------------------------------------------------ worker loop
// The workers walk the program in order. GEMM phases: the epilogue warps
// handle this CTA's segments as their accumulators complete. Attention: this
// CTA's items, each after its inputs. Per-lane phases: this CTA's lanes, after
// the phase's inputs are complete. No CTA waits for phases it does not consume.
// s_flag[0..1]: epilogue broadcasts; [2]: worker go flag; [3]: GEMM phase ok.
template <int BN, int HD>
__device__ void stk_workers(const StackParams& P, uint8_t* work, uint32_t accf0, uint32_t acce0,
                            uint32_t tmem, volatile int* abort_, int* s_flag, float* red) {
  const int wt = threadIdx.x - kStkWorkerTid0;
  if (wt == 0) stk_trace(P, P.n_phases, 0);
  pdl_wait();
  // Co-residency: every CTA of the grid must be running before phases start.
  if (wt == 0) {
    atomicAdd(P.sync, 1u);
    s_flag[2] = grid_wait(P.sync, gridDim.x, abort_, P.err, kDevNotResident, kStkStartNs);
    stk_trace(P, P.n_phases, 1);
  }
  named_bar(kBarWorkers, kStkWorkers);
  if (!s_flag[2]) return;
  int seg = 0;
  for (int p = 0; p < P.n_phases; ++p) {
    const Phase& ph = P.phases[p];
    if (p == P.n_phases - 1) pdl_launch_dependents();
    if (wt == 0) stk_trace(P, p, 0);
    if (ph.kind == kPhGemm) {
      bool ok = true;
      if (threadIdx.x >= kStkEpiTid0 && threadIdx.x < kStkEpiTid0 + 128)   // warps 4..7 only
        ok = stk_gemm_epilogue<BN>(P, ph, p, seg, accf0, acce0, tmem, abort_, s_flag);
      if (threadIdx.x == kStkEpiTid0) s_flag[3] = ok;
      named_bar(kBarWorkers, kStkWorkers);
      if (!s_flag[3]) return;
    } else if (ph.kind == kPhAttn) {
      if (!stk_attention<HD>(P, ph, p, work, abort_, s_flag, !ActPath<BN>::kLdg)) return;
    } else if ((int)blockIdx.x < P.n) {
      if (wt == 0) s_flag[2] = wait_tot_deps(P, ph, abort_);
      named_bar(kBarWorkers, kStkWorkers);
      if (!s_flag[2]) return;
      if (wt == 0) stk_trace(P, p, 2);   // inputs complete
      for (int b = blockIdx.x; b < P.n; b += gridDim.x) {
        switch (ph.kind) {
          case kPhMap: stk_map(P, b); break;
          case kPhPrep: stk_prep(P, ph, b, red); break;
          case kPhCat: stk_cat(P, b); break;
          case kPhQkNorm: stk_qknorm(P, ph, b, red); break;
          case kPhRow: stk_row(P, ph, b, red, p); break;
          case kPhRavenInit: stk_raven_init(P, b); break;
          default:
            if (wt == 0) atomicExch(P.err, kDevBadIndex);
            break;
        }
        if (wt == 0 && b == (int)blockIdx.x) stk_trace(P, p, 4);   // first lane's work done
        const long long cpub = clock64();
        publish(kBarWorkers, kStkWorkers, wt == 0, P.tot + p, nullptr, !ActPath<BN>::kLdg);
        if (wt == 0 && b == (int)blockIdx.x && blockIdx.x == 0)
          stk_trace_value(P, p, 10, (unsigned long long)(clock64() - cpub));   // publish cycles
      }
    }
    if (wt == 0) stk_trace(P, p, 1);
  }
}

template <int BN, int ST, int HD>
__global__ void __launch_bounds__(kStkThreads, 1) stack_kernel(const __grid_constant__ StackLaunch L) {
  using S = StkSmem<BN, ST>;
  const StackParams& P = L.P;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* work = smem + S::kRing;
  uint64_t* bars = reinterpret_cast<uint64_t*>(work + S::kWork);
  const uint32_t full0 = smem_u32(bars), empty0 = full0 + 8 * ST, accf0 = empty0 + 8 * ST;
  const uint32_t acce0 = accf0 + 16, fin = acce0 + 16;
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort_word;
  __shared__ long long s_iw_word;
  __shared__ int s_wdone_word;
  __shared__ int s_flag[4];
  __shared__ float s_red[8];
  volatile int* abort_ = &s_abort_word;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < ST; ++s) {
      mbar_init(full0 + 8 * s, ActPath<BN>::kLdg ? 2 : 1);   // weights (+ the activation warp)
      mbar_init(empty0 + 8 * s, 1);
    }
    mbar_init(accf0, 1);
    mbar_init(accf0 + 8, 1);
    mbar_init(acce0, 128);
    mbar_init(acce0 + 8, 128);
    mbar_init(fin, 1);
    fence_barrier_init();
    *abort_ = 0;
    s_iw_word = 0;
    s_wdone_word = 0;
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&s_tmem), S::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;
  volatile long long* s_iw = &s_iw_word;
  volatile int* s_wdone = &s_wdone_word;
  if (warp == 0) {
    if (lane == 0) stk_weights<BN, ST>(L, smem, full0, empty0, abort_, s_iw, s_wdone);
    __syncwarp();
  } else if (warp == 2) {
    if constexpr (ActPath<BN>::kLdg) {
      stk_acts_ldg<BN, ST>(L, smem, full0, abort_, s_iw, s_wdone);
    } else {
      if (lane == 0) stk_acts<BN, ST>(L, smem, full0, abort_, s_iw, s_wdone);
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) stk_mma<BN, ST>(P, smem, full0, empty0, accf0, acce0, fin, tmem, abort_);
    __syncwarp();
  } else {
    stk_workers<BN, HD>(P, work, accf0, acce0, tmem, abort_, s_flag, s_red);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, S::kTmemCols);
  }
  // The last CTA out resets every counter for the next launch (all other
  // CTAs have finished reading them).
  if (threadIdx.x == 0) {
    __threadfence();
    s_flag[0] = atomicAdd(P.sync + 2, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (s_flag[0]) {
    __threadfence();
    for (int i = threadIdx.x; i < P.n_cnt; i += blockDim.x) P.cnt[i] = 0;
    for (int i = threadIdx.x; i < P.n_phases; i += blockDim.x) P.tot[i] = 0;
    if (threadIdx.x == 0) {
      P.sync[0] = 0;
      P.sync[2] = 0;
    }
    __threadfence();
  }
}

}  // namespace ls
