// Per-lane kernels of one role call: timeline mapping update, state gathers,
// fused split-K reductions with RMSNorm / residual / RoPE / SwiGLU epilogues,
// branch-timeline-aware paged decode attention, and greedy argmax.
//
// Every kernel processes each lane (decode token replica) in its own CTA or
// CTA set with a reduction order that depends only on that lane's data, so a
// lane's numbers do not depend on the batch it runs in (LoopSpec == AR).
// A lane whose metadata position is -1 is inactive (the device-resident loop
// runs every role call at a fixed width): per-lane kernels skip it.
#pragma once

#include "common.cuh"

namespace ls {

// ----------------------------------------------------------- mapping update
// Fork: row[0:fork_len) = parent_row[0:fork_len) (O(fork_len), once per fork),
// then row[pos] = slot. Mirrors the reference's in-graph mapping update
// (sglang_recurrent/loopspec/graph_ops.py:175-218) without its O(context) grid.
__global__ void map_update_kernel(Meta meta, int B, int* __restrict__ map, int max_ctx, int rows,
                                  int* err) {
  pdl_launch_dependents();
  pdl_wait();
  const int b = blockIdx.x;
  if (b >= B || meta.get(kMetaPos, b) < 0) return;   // inactive lane
  const int row = meta.get(kMetaRow, b), pos = meta.get(kMetaPos, b);
  const int frow = meta.get(kMetaForkRow, b), flen = meta.get(kMetaForkLen, b);
  if (row < 0 || row >= rows || pos < 0 || pos >= max_ctx) {
    if (threadIdx.x == 0) atomicExch(err, kDevBadIndex);
    return;
  }
  int* dst = map + (long)row * max_ctx;
  if (frow >= 0) {
    if (frow >= rows || flen > max_ctx) {
      if (threadIdx.x == 0) atomicExch(err, kDevBadIndex);
      return;
    }
    const int* src = map + (long)frow * max_ctx;
    for (int j = threadIdx.x; j < flen; j += blockDim.x) dst[j] = src[j];
  }
  if (threadIdx.x == 0) dst[pos] = meta.get(kMetaSlot, b);
}

// ------------------------------------------------------------- input prep
// h[b] = source row (embedding * scale, or state bank row); optional bank
// write; x[b] = (hi, lo) of (norm ? rms(h) * w : h).
struct PrepArgs {
  Meta meta;
  int B, H;
  const __nv_bfloat16* embed;  // non-null: embed mode
  float embed_scale;
  const float* bank_in;        // gather mode source (indexed by state_in)
  int bank_rows;
  float* h;                    // [cap][H]
  float* bank_out;             // optional: also write h to bank_out[state_out]
  __nv_bfloat16* x;            // optional
  const __nv_bfloat16* x_norm_w;
  float eps;
  int vocab;
  int* err;
  int meta_after_wait;         // the lane metadata comes from the kernel before this one
};

template <int NV>
__global__ void prep_kernel(PrepArgs a) {
  // with metadata written by the preceding kernel, nothing is read and no
  // dependent starts (its pre-wait reads take the metadata) before the wait
  if (a.meta_after_wait) pdl_wait();
  pdl_launch_dependents();
  const int b = blockIdx.x;
  if (b >= a.B || a.meta.get(kMetaPos, b) < 0) return;   // inactive lane
  __shared__ float red[32];
  const int H = a.H, H4 = H / 4;
  int src;
  if (a.embed) {
    src = a.meta.get(kMetaToken, b);
    if (src < 0 || src >= a.vocab) src = -1;
  } else {
    src = a.meta.get(kMetaStateIn, b);
    if (src < 0 || src >= a.bank_rows) src = -1;
  }
  if (src < 0 && threadIdx.x == 0) atomicExch(a.err, kDevBadIndex);
  // The lane metadata is uploaded before the role call and the embedding
  // table and norm weights are constant: load them before waiting on the
  // preceding kernel; a state-bank row only after it.
  float4 v[NV], w[NV];
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int j = threadIdx.x + k * blockDim.x;
    v[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    w[k] = make_float4(1.f, 1.f, 1.f, 1.f);
    if (j < H4 && src >= 0 && a.embed) {
      const float4 e = ld_bf4(a.embed + (long)src * H + 4 * j);
      v[k] = make_float4(e.x * a.embed_scale, e.y * a.embed_scale, e.z * a.embed_scale,
                         e.w * a.embed_scale);
    }
    if (j < H4 && a.x_norm_w) w[k] = ld_bf4(a.x_norm_w + 4 * j);
  }
  pdl_wait();
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int j = threadIdx.x + k * blockDim.x;
    if (j < H4 && src >= 0 && !a.embed) v[k] = ld_f4(a.bank_in + (long)src * H + 4 * j);
    ss += f4_sq(v[k]);
  }
  const int so = a.bank_out ? a.meta.get(kMetaStateOut, b) : -1;
  float inv = 1.f;
  if (a.x && a.x_norm_w) inv = rsqrtf(block_sum(ss, red) / H + a.eps);
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int j = threadIdx.x + k * blockDim.x;
    if (j >= H4) continue;
    *reinterpret_cast<float4*>(a.h + (long)b * H + 4 * j) = v[k];
    if (so >= 0 && so < a.bank_rows) *reinterpret_cast<float4*>(a.bank_out + (long)so * H + 4 * j) = v[k];
    if (a.x) store_pair4(a.x, H, b, 4 * j, a.x_norm_w ? f4_scale(v[k], inv, w[k]) : v[k]);
  }
}

// Raven recurrent input: x[b] = (hi, lo) of [bank_h[state_in], bank_inj[state_in]].
__global__ void cat_state_kernel(Meta meta, int H, const float* __restrict__ bank_h,
                                 const float* __restrict__ bank_inj, int bank_rows,
                                 __nv_bfloat16* __restrict__ x, int* err) {
  pdl_launch_dependents();
  pdl_wait();
  const int b = blockIdx.x;
  if (meta.get(kMetaPos, b) < 0) return;   // inactive lane
  const int si = meta.get(kMetaStateIn, b);
  if (si < 0 || si >= bank_rows) {
    if (threadIdx.x == 0) atomicExch(err, kDevBadIndex);
    return;
  }
  for (int j = threadIdx.x; j < H / 4; j += blockDim.x) {
    const float4 h = ld_f4(bank_h + (long)si * H + 4 * j);
    const float4 g = ld_f4(bank_inj + (long)si * H + 4 * j);
    store_pair4(x, 2L * H, b, 4 * j, h);
    store_pair4(x, 2L * H, b, H + 4 * j, g);
  }
}

// --------------------------------------------------------- tensor parallel
// The ranks of a tensor-parallel group hold 1/T of the heads and of the MLP
// columns each. They exchange partial rows through memory every rank has
// mapped from its peers (CUDA IPC): the O and down projections' split planes,
// and the per-lane sums of squares of OLMo2's QK-norm. A rank publishes an
// exchange by advancing its epoch counter and raising its flag for the
// exchange's slot to the new epoch. A consumer waits (bounded) until every
// rank's flag for that slot has reached its own epoch, then reads all ranks'
// partials in rank order, so every rank computes bit-identical rows. The
// producer does not overwrite a published buffer before every consumer has
// read it: a rank writes a slot's buffer again only after it has consumed
// the next exchange, which each peer publishes after its last read of the
// buffer.
constexpr int kTpMax = 8;
constexpr int kTpSlotO = 0, kTpSlotDown = 1, kTpSlotQk = 2, kTpSlots = 3;
constexpr unsigned long long kTpWaitNs = 10000000000ull;   // default limit per exchange: 10 s

struct TpView {
  int ranks;                    // > 1: this kernel adds the peers' partials
  const int* epoch;             // this rank's exchange counter
  const int* flags[kTpMax];     // each rank's flags [kTpSlots], in rank order
  const float* data[kTpMax];    // each rank's buffer of this exchange
  unsigned long long wait_ns;   // give up on a peer after this long
};

__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Thread 0 waits for every rank's flag of `slot` to reach this rank's epoch.
// Returns false for the whole CTA when the wait gave up (error recorded, or
// another kernel had already recorded one).
__device__ bool tp_wait(const TpView& t, int slot, int* err) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    const int want = ld_volatile(t.epoch);
    const unsigned long long t0 = gtime_ns();
    int good = 1;
    for (int r = 0; r < t.ranks && good; ++r) {
      for (uint32_t i = 0; ld_acquire_sys(t.flags[r] + slot) < want; ++i) {
        if ((i & 63u) == 63u && (ld_volatile(err) != 0 || gtime_ns() - t0 > t.wait_ns)) {
          if (ld_volatile(err) == 0) atomicExch(err, kDevTimeoutPeer);
          good = 0;
          break;
        }
        __nanosleep(32);
      }
    }
    ok = good;
  }
  __syncthreads();
  return ok != 0;
}

// Publish this rank's partials of one exchange once the producing kernel has
// completed: advance the epoch and raise this rank's flag of `slot` to it.
__global__ void tp_publish_kernel(int* epoch, int* flags, int slot) {
  pdl_launch_dependents();
  pdl_wait();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const int e = atomicAdd(epoch, 1) + 1;   // (the O / down GEMMs advance it the same way)
    st_release_sys(flags + slot, e);
  }
}

// ------------------------------------------------------- residual epilogue
// a = y[b] (+ bias); a = a_norm ? rms(a) * wa : a;
// out = (resid ? resid : 0) + a; out = final_norm ? rms(out) * wf : out;
// out_h[b] = out; bank[state_out] = out (optional);
// x[b] = (hi, lo) of (x_norm ? rms(out) * wx : out) (optional).
struct ResidArgs {
  Meta meta;
  int B, H;                    // lanes, hidden size
  const float* part;           // GEMM output y: split planes [splits][cap][H]
  int splits;                  // planes to add, in split order (>= 1)
  long split_stride;           // floats between planes
  const __nv_bfloat16* bias;
  const __nv_bfloat16* a_norm_w;
  const float* resid;
  float* out_h;
  const __nv_bfloat16* final_norm_w;
  float* bank;
  int bank_rows;
  __nv_bfloat16* x;
  const __nv_bfloat16* x_norm_w;
  float eps;
  int* err;
  TpView tp;                   // ranks > 1: y = every rank's planes, rank by rank
  int tp_slot;
};

// NV float4 columns per thread; BATCH split planes loaded at once (one round
// trip for the usual 19 splits when BATCH = 20); MAXT threads at most, which
// bounds the registers the batch may use. TP: add every rank's planes (a
// separate instantiation, so the single-GPU kernel carries none of it).
template <int NV, int BATCH, int MAXT, bool TP>
__global__ void __launch_bounds__(MAXT) resid_epi_kernel(ResidArgs a) {
  pdl_launch_dependents();
  const int b = blockIdx.x;
  if (b >= a.B || a.meta.get(kMetaPos, b) < 0) return;   // inactive lane
  __shared__ float red[32];
  const int H = a.H, H4 = H / 4;
  const float4 z = make_float4(0.f, 0.f, 0.f, 0.f), one = make_float4(1.f, 1.f, 1.f, 1.f);
  float4 v[NV], rr[NV], wa[NV], wf[NV], wx[NV], bb[NV];
  // The norm weights and the bias are constant: load them while the
  // producing GEMM is still running, the rows after it has finished.
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int j = threadIdx.x + k * blockDim.x;
    const bool on = j < H4;
    wa[k] = on && a.a_norm_w ? ld_bf4(a.a_norm_w + 4 * j) : one;
    wf[k] = on && a.final_norm_w ? ld_bf4(a.final_norm_w + 4 * j) : one;
    wx[k] = on && a.x_norm_w ? ld_bf4(a.x_norm_w + 4 * j) : one;
    bb[k] = on && a.bias ? ld_bf4(a.bias + 4 * j) : z;
  }
  pdl_wait();
  if (TP && !tp_wait(a.tp, a.tp_slot, a.err)) return;
  const int n_src = TP ? a.tp.ranks : 1;
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int j = threadIdx.x + k * blockDim.x;
    const bool on = j < H4;
    rr[k] = on && a.resid ? ld_f4(a.resid + (long)b * H + 4 * j) : z;
    // y = the GEMM's split planes added in split order (rank by rank under
    // tensor parallelism; peers' planes over NVLink), BATCH loads in flight
    v[k] = z;
    if (on) {
      for (int src = 0; src < n_src; ++src) {
        const float* py = (TP ? a.tp.data[src] : a.part) + (long)b * H + 4 * j;
        for (int s0 = 0; s0 < a.splits; s0 += BATCH) {
          float4 t[BATCH];
#pragma unroll
          for (int u = 0; u < BATCH; ++u)
            if (s0 + u < a.splits) t[u] = TP ? ldcg4(py + (s0 + u) * a.split_stride)
                                             : ld_f4(py + (s0 + u) * a.split_stride);
#pragma unroll
          for (int u = 0; u < BATCH; ++u)
            if (s0 + u < a.splits)
              v[k] = make_float4(v[k].x + t[u].x, v[k].y + t[u].y, v[k].z + t[u].z, v[k].w + t[u].w);
        }
      }
    }
    if (a.bias) v[k] = make_float4(v[k].x + bb[k].x, v[k].y + bb[k].y, v[k].z + bb[k].z, v[k].w + bb[k].w);
    ss += f4_sq(v[k]);
  }
  const int so = a.bank ? a.meta.get(kMetaStateOut, b) : -1;
  if (a.a_norm_w) {
    const float inv = rsqrtf(block_sum(ss, red) / H + a.eps);
#pragma unroll
    for (int k = 0; k < NV; ++k) v[k] = f4_scale(v[k], inv, wa[k]);
  }
  ss = 0.f;
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    v[k] = make_float4(v[k].x + rr[k].x, v[k].y + rr[k].y, v[k].z + rr[k].z, v[k].w + rr[k].w);
    ss += f4_sq(v[k]);
  }
  if (a.final_norm_w) {
    const float inv = rsqrtf(block_sum(ss, red) / H + a.eps);
    ss = 0.f;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      v[k] = f4_scale(v[k], inv, wf[k]);
      ss += f4_sq(v[k]);
    }
  }
  float inv = 1.f;
  if (a.x && a.x_norm_w) inv = rsqrtf(block_sum(ss, red) / H + a.eps);
  if (a.bank && (so < 0 || so >= a.bank_rows) && threadIdx.x == 0) atomicExch(a.err, kDevBadIndex);
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int j = threadIdx.x + k * blockDim.x;
    if (j >= H4) continue;
    *reinterpret_cast<float4*>(a.out_h + (long)b * H + 4 * j) = v[k];
    if (a.bank && so >= 0 && so < a.bank_rows)
      *reinterpret_cast<float4*>(a.bank + (long)so * H + 4 * j) = v[k];
    if (a.x) store_pair4(a.x, H, b, 4 * j, a.x_norm_w ? f4_scale(v[k], inv, wx[k]) : v[k]);
  }
}

// ------------------------------------------------------------- QKV epilogue
// Split-sum the fused QKV projection of lane b, apply the optional OLMo2
// QK-norm (RMSNorm over the whole q and k projections), neox RoPE at the
// lane's position, write K and V (bf16) into this layer's KV pool at the
// lane's slot, and keep q (fp32) for attention.
struct QkvArgs {
  Meta meta;
  int nh, nkv, hd;
  const float* part;
  int splits;
  long split_stride;
  const __nv_bfloat16* q_norm_w;   // optional
  const __nv_bfloat16* k_norm_w;
  const float* inv_freq;           // [hd/2]
  float eps;
  float* q;                        // [cap][nh*hd]
  __nv_bfloat16* kpool;            // this layer's [slots][nkv*hd]
  __nv_bfloat16* vpool;
  int n_slots;
  int* err;
  // Tensor parallel QK-norm (q_norm_w set, tp.ranks > 1): phase 1 writes this
  // rank's (sum q^2, sum k^2) of each lane to tp_sums and returns; phase 2
  // adds every rank's sums in rank order and normalises by the whole width.
  TpView tp;
  int tp_phase;
  float* tp_sums;   // this rank's [cap][2]
};

__global__ void qkv_epi_kernel(QkvArgs a) {
  pdl_launch_dependents();
  pdl_wait();
  extern __shared__ float row[];
  __shared__ float red[32];
  const int b = blockIdx.x;
  if (a.meta.get(kMetaPos, b) < 0) return;   // inactive lane
  const int qd = a.nh * a.hd, kd = a.nkv * a.hd, D = qd + 2 * kd;
  const bool tp = a.q_norm_w && a.tp.ranks > 1;
  if (tp && a.tp_phase == 2 && !tp_wait(a.tp, kTpSlotQk, a.err)) return;
  const float* pb = a.part + (long)b * D;
  float ssq = 0.f, ssk = 0.f;
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    float v = pb[i];
    for (int s = 1; s < a.splits; ++s) v += pb[(long)s * a.split_stride + i];
    row[i] = v;
    if (i < qd) ssq += v * v;
    else if (i < qd + kd) ssk += v * v;
  }
  if (tp && a.tp_phase == 1) {
    ssq = block_sum(ssq, red);
    ssk = block_sum(ssk, red);
    if (threadIdx.x == 0) {
      a.tp_sums[2L * b] = ssq;
      a.tp_sums[2L * b + 1] = ssk;
    }
    return;
  }
  if (tp) {
    ssq = 0.f;
    ssk = 0.f;
    for (int r = 0; r < a.tp.ranks; ++r) {
      ssq += __ldcg(a.tp.data[r] + 2L * b);
      ssk += __ldcg(a.tp.data[r] + 2L * b + 1);
    }
    const float iq = rsqrtf(ssq / ((float)qd * a.tp.ranks) + a.eps);
    const float ik = rsqrtf(ssk / ((float)kd * a.tp.ranks) + a.eps);
    for (int i = threadIdx.x; i < qd + kd; i += blockDim.x)
      row[i] = i < qd ? row[i] * iq * bf2f(a.q_norm_w[i]) : row[i] * ik * bf2f(a.k_norm_w[i - qd]);
  } else if (a.q_norm_w) {
    const float iq = rsqrtf(block_sum(ssq, red) / qd + a.eps);
    const float ik = rsqrtf(block_sum(ssk, red) / kd + a.eps);
    for (int i = threadIdx.x; i < qd + kd; i += blockDim.x)
      row[i] = i < qd ? row[i] * iq * bf2f(a.q_norm_w[i]) : row[i] * ik * bf2f(a.k_norm_w[i - qd]);
  }
  __syncthreads();
  const int pos = a.meta.get(kMetaPos, b);
  const int slot = a.meta.get(kMetaSlot, b);
  const bool slot_ok = slot >= 0 && slot < a.n_slots;
  if (!slot_ok && threadIdx.x == 0) atomicExch(a.err, kDevBadIndex);
  const int half = a.hd / 2;
  const int pairs = (a.nh + a.nkv) * half;
  const float fpos = (float)pos;
  for (int t = threadIdx.x; t < pairs; t += blockDim.x) {
    const int head = t / half, i = t - head * half;
    const int base = head * a.hd;
    const float x1 = row[base + i], x2 = row[base + i + half];
    float sn, cs;
    sincosf(fpos * a.inv_freq[i], &sn, &cs);
    const float y1 = x1 * cs - x2 * sn, y2 = x2 * cs + x1 * sn;
    if (head < a.nh) {
      a.q[(long)b * qd + base + i] = y1;
      a.q[(long)b * qd + base + i + half] = y2;
    } else if (slot_ok) {
      __nv_bfloat16* kr = a.kpool + (long)slot * kd + (base - qd);
      kr[i] = f2bf(y1);
      kr[i + half] = f2bf(y2);
    }
  }
  if (slot_ok) {
    __nv_bfloat16* vr = a.vpool + (long)slot * kd;
    for (int i = threadIdx.x; i < kd; i += blockDim.x) vr[i] = f2bf(row[qd + kd + i]);
  }
}

// ---------------------------------------------------------------- attention
// One CTA per (lane, kv head, chunk of kAttnChunk positions). The lane's
// timeline is its mapping row: position j of the timeline lives in KV slot
// map[row][j], so forked branches read their shared prefix through the same
// slots as their parent. A group of G = nh/nkv query heads shares each K/V
// row. The chunk's slot ids and the query are loaded together; then each
// sub-group of HD/8 threads owns PER fixed positions and issues all of its
// 16-byte K and V loads at once, so a CTA costs two dependent memory round
// trips before its partial; several CTAs per SM overlap theirs. Scores are
// reduced with warp shuffles. Chunk boundaries are fixed multiples of
// kAttnChunk and positions map to sub-groups by index, so results do not
// depend on the batch. Each CTA writes its unnormalised (acc, max, sum)
// partial; the last CTA of a (lane, kv head) to finish (atomic ticket, then
// reset) merges the chunks in chunk order, eight at a time with a running
// max, and writes the attention output as the O GEMM's bf16 (hi, lo) input.
constexpr int kAttnChunk = 128;
constexpr int kAttnThreads = 256;
constexpr int kAttnMaxChunks = 1024;   // max_context <= 131072

struct AttnArgs {
  Meta meta;
  int nh, nkv;
  const float* q;                  // [cap][nh*HD]
  const int* map;
  int max_ctx, rows;
  const __nv_bfloat16* kpool;      // this layer's [slots][nkv*HD]
  const __nv_bfloat16* vpool;
  int n_slots;
  int max_chunks;
  float* o_part;                   // [cap][nh][max_chunks][HD]
  float* ml_part;                  // [cap][nh][max_chunks][2]
  int* tickets;                    // [cap][nkv], zero between calls
  __nv_bfloat16* x;                // (hi, lo) rows [2*cap][nh*HD], or
  float* out;                      // ... fp32 rows [cap][nh*HD] when non-null
  const int* lane_len;             // optional per-lane timeline length (else pos + 1)
  const int* lane_row;             // optional per-lane mapping row (else metadata)
  float scale;
  int* err;
  // Decode form (qkv non-null): the QKV projection left its split planes
  // [splits][cap][(nh + 2 nkv) * HD] and every lane has exactly one new
  // position (T - 1). Each CTA sums its q (split order) and applies RoPE; the
  // CTA whose chunk holds T - 1 also forms that position's K (RoPE) and V,
  // rounds them to bf16, writes them to the pool at the position's slot and
  // uses them.
  const float* qkv;
  int qkv_splits;
  long qkv_stride;
  const float* inv_freq;           // [HD / 2]
  __nv_bfloat16* kpool_w;          // kpool / vpool, writable
  __nv_bfloat16* vpool_w;
};

// Sum of `splits` planes of element e (split order) starting at p.
__device__ __forceinline__ float plane_sum(const float* p, int splits, long stride) {
  float t[8], v = 0.f;
  for (int s0 = 0; s0 < splits; s0 += 8) {
#pragma unroll
    for (int u = 0; u < 8; ++u) t[u] = s0 + u < splits ? __ldcg(p + (s0 + u) * stride) : 0.f;
#pragma unroll
    for (int u = 0; u < 8; ++u)
      if (s0 + u < splits) v += t[u];
  }
  return v;
}

// Register budget by grid size (same arithmetic in every form):
//   kAttnWide  (<= 1 CTA per SM): K and V before the wait, 2 CTAs' registers
//              per SM, no spills;
//   kAttnMid   (<= 2 CTAs per SM): K and V before the wait, 3 per SM;
//   kAttnVLate (larger grids): only K before the wait into registers, V of
//              the older positions copied to shared memory (cp.async) before
//              the wait and read after the scores into K's registers; 4 CTAs
//              per SM.
enum AttnForm : int { kAttnWide = 0, kAttnMid = 1, kAttnVLate = 2 };

template <int HD, int G, int FORM>
__global__ void __launch_bounds__(kAttnThreads, FORM + 2) attn_kernel(AttnArgs a) {
  constexpr bool VLATE = FORM == kAttnVLate;
  pdl_launch_dependents();
  constexpr int LPP = HD / 8;              // lanes per position (16 B each)
  constexpr int PPW = 32 / LPP;            // positions per warp at a time
  constexpr int NW = kAttnThreads / 32;
  constexpr int NSG = NW * PPW;            // sub-groups per CTA
  constexpr int PER = kAttnChunk / NSG;    // positions per sub-group
  static_assert(PER * NSG == kAttnChunk, "chunk must split evenly over sub-groups");
  // Before waiting on the preceding kernel (the QKV projection that writes q
  // and the newest position's K/V), load what earlier work wrote: the lane
  // metadata (uploaded before the role call), the timeline's slot ids of the
  // positions older than this call and the K/V rows of those positions. A
  // call whose mapping update appends several positions per timeline
  // (prefill) launches the kernel after the update without programmatic
  // overlap, so those entries are final before this kernel starts;
  // otherwise the update copies forked prefixes (read here from the parent's
  // row) and appends each lane's new position, which this kernel takes from
  // the metadata.
  const int b = blockIdx.x, g = blockIdx.y, c = blockIdx.z;
  if (!a.lane_len && a.meta.get(kMetaPos, b) < 0) return;   // inactive lane
  const int T = a.lane_len ? a.lane_len[b] : a.meta.get(kMetaPos, b) + 1;
  // the grid holds one CTA per chunk of the call's longest timeline
  if (T < 1 || T > a.max_ctx || (T + kAttnChunk - 1) / kAttnChunk > (int)gridDim.z) {
    if (threadIdx.x == 0 && c == 0) atomicExch(a.err, kDevBadIndex);
    return;
  }
  const int start = c * kAttnChunk;
  if (start >= T) return;
  const int n_in = min(kAttnChunk, T - start);
  const int row = a.lane_row ? a.lane_row[b] : a.meta.get(kMetaRow, b);
  if (row < 0 || row >= a.rows) {
    if (threadIdx.x == 0) atomicExch(a.err, kDevBadIndex);
    return;
  }
  __shared__ int s_slot[kAttnChunk];
  __shared__ float s_raw[G * HD + 2 * HD];               // decode form: plane sums
  __shared__ float s_q[G * HD];                          // decode form: q after RoPE
  __shared__ __align__(16) __nv_bfloat16 s_kv[2 * HD];   // decode form: new K, V (bf16)
  __shared__ float sm_m[NW][G], sm_l[NW][G];
  __shared__ float sm_acc[NW][G][HD];
  __shared__ int s_last;
  // late-V form: each thread's V rows of positions older than this call,
  // staged by cp.async before the wait (registers stay K's only)
  __shared__ __align__(16) uint4 s_v[VLATE ? PER : 1][VLATE ? kAttnThreads : 1];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sub = lane / LPP, sl = lane % LPP;
  const int sg = warp * PPW + sub;
  const int kd = a.nkv * HD;

  // decode form: RoPE angles of position T - 1 (they depend on nothing the
  // preceding kernel writes)
  __shared__ float s_cs[HD / 2], s_sn[HD / 2];
  if (a.qkv && threadIdx.x < HD / 2) sincosf((float)(T - 1) * a.inv_freq[threadIdx.x], &s_sn[threadIdx.x], &s_cs[threadIdx.x]);
  // chunk index of the first position written by this call (the QKV
  // projection writes one position per lane; prefill puts several positions
  // of one timeline in a call)
  const int fresh = T - 1 - (a.lane_len ? 0 : a.meta.get(kMetaAhead, b)) - start;
  // a lane whose timeline this call forks has its prefix copied into its
  // mapping row by the call's mapping update, which may still be running:
  // positions of the prefix are read from the parent's row, whose entries
  // earlier calls wrote
  const int frow = a.lane_len ? -1 : a.meta.get(kMetaForkRow, b);
  const int flen = frow >= 0 && frow < a.rows ? a.meta.get(kMetaForkLen, b) : 0;
  int sv = -1;
  if (threadIdx.x < kAttnChunk && (int)threadIdx.x < n_in) {
    // decode form: the new position's slot comes from the lane metadata, so
    // its mapping entry (appended by this call's mapping update) is never read
    const int t = start + threadIdx.x;
    sv = a.qkv && (int)threadIdx.x == fresh ? a.meta.get(kMetaSlot, b)
                                            : a.map[(long)(t < flen ? frow : row) * a.max_ctx + t];
  }
  if (threadIdx.x < kAttnChunk) {
    if ((int)threadIdx.x < n_in && (sv < 0 || sv >= a.n_slots)) {
      atomicExch(a.err, kDevBadIndex);
      sv = -1;
    }
    s_slot[threadIdx.x] = sv;
  }
  __syncthreads();
  uint4 kr[PER], vr[PER];
#pragma unroll
  for (int t = 0; t < PER; ++t) {
    const int i = sg + t * NSG;
    const int slot = s_slot[i];
    const long off = (long)slot * kd + g * HD + sl * 8;
    const bool old_row = slot >= 0 && i < fresh;
    kr[t] = old_row ? *reinterpret_cast<const uint4*>(a.kpool + off) : make_uint4(0, 0, 0, 0);
    if (!VLATE) vr[t] = old_row ? *reinterpret_cast<const uint4*>(a.vpool + off) : make_uint4(0, 0, 0, 0);
    else if (old_row) cp_async16(&s_v[t][threadIdx.x], a.vpool + off, true);
  }
  if (VLATE) cp_async_commit();
  pdl_wait();
  // after the QKV projection: this thread's query slice and the newest K/V row
  float qv[G][8];
  if (a.qkv) {
    // decode form: q, and (chunk holding T - 1) the new K/V, from the planes
    constexpr int half = HD / 2;
    const bool own = fresh >= 0 && fresh < kAttnChunk;   // this chunk holds T - 1
    const int D = (a.nh + 2 * a.nkv) * HD;
    const float* pl = a.qkv + (long)b * D;
    const int n_el = G * HD + (own ? 2 * HD : 0);
    for (int e = threadIdx.x; e < n_el; e += blockDim.x) {
      int col;
      if (e < G * HD) col = g * G * HD + e;                                   // q of head g*G + e/HD
      else if (e < G * HD + HD) col = (a.nh + g) * HD + (e - G * HD);         // k of kv head g
      else col = (a.nh + a.nkv + g) * HD + (e - G * HD - HD);                 // v of kv head g
      s_raw[e] = plane_sum(pl + col, a.qkv_splits, a.qkv_stride);
    }
    __syncthreads();
    for (int e = threadIdx.x; e < n_el; e += blockDim.x) {
      if (e < G * HD + HD) {   // q or k: neox RoPE pairs (i, i + half) within a head
        const int base = e < G * HD ? (e / HD) * HD : G * HD;
        const int d = e - base, i = d < half ? d : d - half;
        const float sn = s_sn[i], cs = s_cs[i];
        const float x1 = s_raw[base + i], x2 = s_raw[base + i + half];
        const float y = d < half ? x1 * cs - x2 * sn : x2 * cs + x1 * sn;
        if (e < G * HD) s_q[e] = y;
        else s_kv[d] = f2bf(y);
      } else {
        s_kv[e - G * HD] = f2bf(s_raw[e]);
      }
    }
    __syncthreads();
    if (own) {   // the pool keeps the new K/V for later calls, at the lane's slot
      const int slot = a.meta.get(kMetaSlot, b);
      if (slot < 0 || slot >= a.n_slots) {
        if (threadIdx.x == 0) atomicExch(a.err, kDevBadIndex);
      } else
        for (int e = threadIdx.x; e < 2 * HD; e += blockDim.x)
          (e < HD ? a.kpool_w : a.vpool_w)[(long)slot * kd + g * HD + (e % HD)] = s_kv[e];
    }
#pragma unroll
    for (int h = 0; h < G; ++h)
#pragma unroll
      for (int d = 0; d < 8; ++d) qv[h][d] = s_q[h * HD + sl * 8 + d] * a.scale;
#pragma unroll
    for (int t = 0; t < PER; ++t) {
      const int i = sg + t * NSG;
      if (own && i == fresh && s_slot[i] >= 0) {
        kr[t] = *reinterpret_cast<const uint4*>(s_kv + sl * 8);
        if (!VLATE) vr[t] = *reinterpret_cast<const uint4*>(s_kv + HD + sl * 8);
      }
    }
  } else {
#pragma unroll
    for (int h = 0; h < G; ++h) {
      const float* qp = a.q + (long)b * a.nh * HD + (g * G + h) * HD + sl * 8;
      const float4 q0 = ld_f4(qp), q1 = ld_f4(qp + 4);
      const float qq[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
      for (int d = 0; d < 8; ++d) qv[h][d] = qq[d] * a.scale;
    }
#pragma unroll
    for (int t = 0; t < PER; ++t) {
      const int i = sg + t * NSG;
      const int slot = s_slot[i];
      if (slot >= 0 && i >= fresh) {
        const long off = (long)slot * kd + g * HD + sl * 8;
        kr[t] = *reinterpret_cast<const uint4*>(a.kpool + off);
        if (!VLATE) vr[t] = *reinterpret_cast<const uint4*>(a.vpool + off);
      }
    }
  }
  float sc[G][PER];
#pragma unroll
  for (int t = 0; t < PER; ++t) {
    float kf[8];
    unpack8(kr[t], kf);
#pragma unroll
    for (int h = 0; h < G; ++h) {
      float s = 0.f;
#pragma unroll
      for (int d = 0; d < 8; ++d) s += qv[h][d] * kf[d];
#pragma unroll
      for (int o = LPP / 2; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      sc[h][t] = s_slot[sg + t * NSG] >= 0 ? s : -INFINITY;
    }
  }
  if (VLATE) {   // every V row now: older positions from the staged copies, the new one
                 // (decode form) from s_kv, positions this call wrote otherwise from the pool
    cp_async_wait<0>();
#pragma unroll
    for (int t = 0; t < PER; ++t) {
      const int i = sg + t * NSG;
      const int slot = s_slot[i];
      if (slot < 0) vr[t] = make_uint4(0, 0, 0, 0);
      else if (i < fresh) vr[t] = s_v[t][threadIdx.x];
      else if (a.qkv && i == fresh) vr[t] = *reinterpret_cast<const uint4*>(s_kv + HD + sl * 8);
      else vr[t] = *reinterpret_cast<const uint4*>(a.vpool + (long)slot * kd + g * HD + sl * 8);
    }
  }
  float m[G], l[G], acc[G][8];
#pragma unroll
  for (int h = 0; h < G; ++h) {
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
    for (int h = 0; h < G; ++h) {
      const float p = m[h] == -INFINITY ? 0.f : __expf(sc[h][t] - m[h]);
      l[h] += p;
#pragma unroll
      for (int d = 0; d < 8; ++d) acc[h][d] += p * vf[d];
    }
  }

  // merge sub-groups within the warp, then warps through shared memory
#pragma unroll
  for (int h = 0; h < G; ++h) {
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
      for (int d = 0; d < 8; ++d) sm_acc[warp][h][sl * 8 + d] = acc[h][d];
      if (sl == 0) {
        sm_m[warp][h] = m[h];
        sm_l[warp][h] = l[h];
      }
    }
  }
  __syncthreads();
  for (int t = threadIdx.x; t < G * HD; t += blockDim.x) {
    const int h = t / HD, d = t - h * HD;
    float mm = -INFINITY;
#pragma unroll
    for (int w = 0; w < NW; ++w) mm = fmaxf(mm, sm_m[w][h]);
    float ll = 0.f, aa = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      const float cw = mm == -INFINITY ? 0.f : __expf(sm_m[w][h] - mm);
      ll += sm_l[w][h] * cw;
      aa += sm_acc[w][h][d] * cw;
    }
    const long idx = ((long)b * a.nh + g * G + h) * a.max_chunks + c;
    a.o_part[idx * HD + d] = aa;
    if (d == 0) {
      a.ml_part[idx * 2] = mm;
      a.ml_part[idx * 2 + 1] = ll;
    }
  }

  // last CTA of this (lane, kv head) merges the chunks in order
  const int nch = min((T + kAttnChunk - 1) / kAttnChunk, a.max_chunks);
  __syncthreads();
  if (threadIdx.x == 0) {
    int* tk = a.tickets + (long)b * a.nkv + g;
    const int ticket = ticket_take(tk);
    s_last = ticket == nch - 1;
    if (s_last) *tk = 0;
  }
  __syncthreads();
  if (!s_last) return;
  // L2 loads (other CTAs wrote the partials), eight chunks in flight at a time
  for (int t = threadIdx.x; t < G * HD; t += blockDim.x) {
    const int h = t / HD, d = t - h * HD;
    const long base = ((long)b * a.nh + g * G + h) * a.max_chunks;
    float mm = -INFINITY, ll = 0.f, aa = 0.f;
    for (int c0 = 0; c0 < nch; c0 += 8) {
      float cm[8], cl[8], co[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        cm[j] = -INFINITY;
        cl[j] = 0.f;
        co[j] = 0.f;
        if (c0 + j < nch) {
          const float2 ml = __ldcg(reinterpret_cast<const float2*>(a.ml_part + (base + c0 + j) * 2));
          cm[j] = ml.x;
          cl[j] = ml.y;
          co[j] = __ldcg(a.o_part + (base + c0 + j) * HD + d);
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
    const float o = ll > 0.f ? aa / ll : 0.f;
    if (a.out) a.out[(long)b * a.nh * HD + (g * G + h) * HD + d] = o;
    else store_pair(a.x, (long)a.nh * HD, b, (g * G + h) * HD + d, o);
  }
}

// ------------------------------------------------------------------ argmax
// out[b] = argmax_v logits[b][v], lowest index among equal maxima
// (torch.argmax semantics, sglang_recurrent/loopspec/decisions.py:116).
__global__ void argmax_kernel(const float* __restrict__ logits, int V, long ld,
                              long long* __restrict__ out) {
  pdl_launch_dependents();
  pdl_wait();
  const int b = blockIdx.x;
  const float* r = logits + (long)b * ld;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  auto take = [&](float x, int v) {
    if (x > best || (x == best && v < bi)) {
      best = x;
      bi = v;
    }
  };
  if (((V | ld) & 3) == 0) {
    // 16-byte loads, several in flight per thread (rows are 16-byte aligned)
#pragma unroll 4
    for (int j = threadIdx.x; j < V / 4; j += blockDim.x) {
      const float4 x = *reinterpret_cast<const float4*>(r + 4 * j);
      take(x.x, 4 * j);
      take(x.y, 4 * j + 1);
      take(x.z, 4 * j + 2);
      take(x.w, 4 * j + 3);
    }
  } else {
#pragma unroll 4
    for (int v = threadIdx.x; v < V; v += blockDim.x) take(r[v], v);
  }
  __shared__ float sb[32];
  __shared__ int si[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ob > best || (ob == best && oi < bi)) {
      best = ob;
      bi = oi;
    }
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) {
    sb[warp] = best;
    si[warp] = bi;
  }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    best = lane < nw ? sb[lane] : -INFINITY;
    bi = lane < nw ? si[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ob > best || (ob == best && oi < bi)) {
        best = ob;
        bi = oi;
      }
    }
    if (lane == 0) out[b] = bi == 0x7fffffff ? 0 : bi;
  }
}

// --------------------------------------------------------- Raven state init
// bank_h[state_out] = truncnormal(0, std; +-3 std)(seed, pos) * scale;
// bank_inj[state_out] = h[b] (the prelude output).
__global__ void raven_init_kernel(Meta meta, int H, const float* __restrict__ h,
                                  float* __restrict__ bank_h, float* __restrict__ bank_inj,
                                  int bank_rows, unsigned long long seed, float std_,
                                  float scale, int* err) {
  pdl_launch_dependents();
  pdl_wait();
  const int b = blockIdx.x;
  if (meta.get(kMetaPos, b) < 0) return;   // inactive lane
  const int so = meta.get(kMetaStateOut, b);
  if (so < 0 || so >= bank_rows) {
    if (threadIdx.x == 0) atomicExch(err, kDevBadIndex);
    return;
  }
  const uint32_t pos = (uint32_t)meta.get(kMetaPos, b);
  const double lo = 0.0013498980316300946;  // Phi(-3)
  for (int i4 = threadIdx.x; i4 < (H + 3) / 4; i4 += blockDim.x) {
    const uint4 w = philox4x32_10(make_uint4((uint32_t)i4, pos, 0u, 0u), (uint32_t)seed,
                                  (uint32_t)(seed >> 32));
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int i = i4 * 4 + k;
      if (i >= H) break;
      const double u = ((double)(ws[k] >> 8) + 0.5) / 16777216.0;
      const double p = lo + u * (1.0 - 2.0 * lo);
      const double x = 1.4142135623730951 * erfinv(2.0 * p - 1.0);
      bank_h[(long)so * H + i] = std_ > 0.f ? (float)(x * std_ * scale) : 0.f;
    }
  }
  for (int i = threadIdx.x; i < H; i += blockDim.x) bank_inj[(long)so * H + i] = h[(long)b * H + i];
}

}  // namespace ls
