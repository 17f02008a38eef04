// Per-lane kernels of one role call: timeline mapping update, state gathers,
// fused split-K reductions with RMSNorm / residual / RoPE / SwiGLU epilogues,
// branch-timeline-aware paged decode attention, and greedy argmax.
//
// Every kernel processes each lane (decode token replica) in its own CTA or
// CTA set with a reduction order that depends only on that lane's data, so a
// lane's numbers do not depend on the batch it runs in (LoopSpec == AR).
#pragma once

#include "common.cuh"

namespace ls {

// Lane metadata: int32 [kMetaFields][cap], field-major.
enum MetaField : int {
  kMetaToken = 0,
  kMetaPos = 1,       // sequence position of the lane's input token
  kMetaRow = 2,       // mapping row of the lane's timeline in this role/depth
  kMetaSlot = 3,      // KV slot receiving this token's K/V for this timeline
  kMetaForkRow = 4,   // parent mapping row to copy a prefix from, or -1
  kMetaForkLen = 5,   // prefix length to copy
  kMetaStateIn = 6,   // state-bank row read by this role
  kMetaStateOut = 7,  // state-bank row written by this role
  kMetaFields = 8,
};

struct Meta {
  const int* p;
  int cap;
  __device__ __forceinline__ int get(int f, int b) const { return p[f * cap + b]; }
};

// ----------------------------------------------------------- mapping update
// Fork: row[0:fork_len) = parent_row[0:fork_len) (O(fork_len), once per fork),
// then row[pos] = slot. Mirrors the reference's in-graph mapping update
// (sglang_recurrent/loopspec/graph_ops.py:175-218) without its O(context) grid.
__global__ void map_update_kernel(Meta meta, int B, int* __restrict__ map, int max_ctx, int rows,
                                  int* err) {
  pdl_wait();
  pdl_launch_dependents();
  const int b = blockIdx.x;
  if (b >= B) return;
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
// write; x[b] = bf16(norm ? rms(h) * w : h).
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
};

__global__ void prep_kernel(PrepArgs a) {
  pdl_wait();
  pdl_launch_dependents();
  extern __shared__ float row[];
  __shared__ float red[32];
  const int b = blockIdx.x;
  const int H = a.H;
  int src;
  if (a.embed) {
    src = a.meta.get(kMetaToken, b);
    if (src < 0 || src >= a.vocab) src = -1;
  } else {
    src = a.meta.get(kMetaStateIn, b);
    if (src < 0 || src >= a.bank_rows) src = -1;
  }
  if (src < 0 && threadIdx.x == 0) atomicExch(a.err, kDevBadIndex);
  float ss = 0.f;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    float v = 0.f;
    if (src >= 0) v = a.embed ? bf2f(a.embed[(long)src * H + i]) * a.embed_scale
                              : a.bank_in[(long)src * H + i];
    row[i] = v;
    ss += v * v;
    a.h[(long)b * H + i] = v;
  }
  if (a.bank_out) {
    const int so = a.meta.get(kMetaStateOut, b);
    if (so >= 0 && so < a.bank_rows)
      for (int i = threadIdx.x; i < H; i += blockDim.x) a.bank_out[(long)so * H + i] = row[i];
  }
  if (a.x) {
    float inv = 1.f;
    if (a.x_norm_w) inv = rsqrtf(block_sum(ss, red) / H + a.eps);
    for (int i = threadIdx.x; i < H; i += blockDim.x) {
      float v = row[i];
      if (a.x_norm_w) v = v * inv * bf2f(a.x_norm_w[i]);
      store_pair(a.x, H, b, i, v);
    }
  }
}

// Raven recurrent input: x[b] = [bf16(bank_h[state_in]), bf16(bank_inj[state_in])].
__global__ void cat_state_kernel(Meta meta, int H, const float* __restrict__ bank_h,
                                 const float* __restrict__ bank_inj, int bank_rows,
                                 __nv_bfloat16* __restrict__ x, int* err) {
  pdl_wait();
  pdl_launch_dependents();
  const int b = blockIdx.x;
  const int si = meta.get(kMetaStateIn, b);
  if (si < 0 || si >= bank_rows) {
    if (threadIdx.x == 0) atomicExch(err, kDevBadIndex);
    return;
  }
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    store_pair(x, 2L * H, b, i, bank_h[(long)si * H + i]);
    store_pair(x, 2L * H, b, H + i, bank_inj[(long)si * H + i]);
  }
}

// ------------------------------------------------------- residual epilogue
// a = sum_s part[s][b] (+ bias); a = a_norm ? rms(a) * wa : a;
// out = (resid ? resid : 0) + a; out = final_norm ? rms(out) * wf : out;
// out_h[b] = out; bank[state_out] = out (optional);
// x[b] = bf16(x_norm ? rms(out) * wx : out) (optional).
struct ResidArgs {
  Meta meta;
  int H;
  const float* part;
  int splits;
  long split_stride;
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
};

__global__ void resid_epi_kernel(ResidArgs a) {
  pdl_wait();
  pdl_launch_dependents();
  extern __shared__ float row[];
  __shared__ float red[32];
  const int b = blockIdx.x;
  const int H = a.H;
  const float* pb = a.part + (long)b * H;
  float ss = 0.f;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    float v = pb[i];
    for (int s = 1; s < a.splits; ++s) v += pb[(long)s * a.split_stride + i];
    if (a.bias) v += bf2f(a.bias[i]);
    row[i] = v;
    ss += v * v;
  }
  if (a.a_norm_w) {
    const float inv = rsqrtf(block_sum(ss, red) / H + a.eps);
    for (int i = threadIdx.x; i < H; i += blockDim.x) row[i] = row[i] * inv * bf2f(a.a_norm_w[i]);
  }
  ss = 0.f;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    float v = row[i];
    if (a.resid) v += a.resid[(long)b * H + i];
    row[i] = v;
    ss += v * v;
  }
  if (a.final_norm_w) {
    const float inv = rsqrtf(block_sum(ss, red) / H + a.eps);
    ss = 0.f;
    for (int i = threadIdx.x; i < H; i += blockDim.x) {
      const float v = row[i] * inv * bf2f(a.final_norm_w[i]);
      row[i] = v;
      ss += v * v;
    }
  }
  for (int i = threadIdx.x; i < H; i += blockDim.x) a.out_h[(long)b * H + i] = row[i];
  if (a.bank) {
    const int so = a.meta.get(kMetaStateOut, b);
    if (so >= 0 && so < a.bank_rows) {
      for (int i = threadIdx.x; i < H; i += blockDim.x) a.bank[(long)so * H + i] = row[i];
    } else if (threadIdx.x == 0) {
      atomicExch(a.err, kDevBadIndex);
    }
  }
  if (a.x) {
    float inv = 1.f;
    if (a.x_norm_w) inv = rsqrtf(block_sum(ss, red) / H + a.eps);
    for (int i = threadIdx.x; i < H; i += blockDim.x) {
      float v = row[i];
      if (a.x_norm_w) v = v * inv * bf2f(a.x_norm_w[i]);
      store_pair(a.x, H, b, i, v);
    }
  }
}

// ------------------------------------------------------------ SwiGLU epilogue
// x[b][i] = bf16(silu(g) * u), g/u = split-summed halves of the gate_up output.
__global__ void act_epi_kernel(const float* __restrict__ part, int splits, long split_stride,
                               int I, __nv_bfloat16* __restrict__ x) {
  pdl_wait();
  pdl_launch_dependents();
  const int b = blockIdx.y;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= I) return;
  const float* pb = part + (long)b * 2 * I;
  float g = pb[i], u = pb[I + i];
  for (int s = 1; s < splits; ++s) {
    g += pb[(long)s * split_stride + i];
    u += pb[(long)s * split_stride + I + i];
  }
  const float sg = g / (1.f + expf(-g));
  store_pair(x, I, b, i, sg * u);
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
};

__global__ void qkv_epi_kernel(QkvArgs a) {
  pdl_wait();
  pdl_launch_dependents();
  extern __shared__ float row[];
  __shared__ float red[32];
  const int b = blockIdx.x;
  const int qd = a.nh * a.hd, kd = a.nkv * a.hd, D = qd + 2 * kd;
  const float* pb = a.part + (long)b * D;
  float ssq = 0.f, ssk = 0.f;
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    float v = pb[i];
    for (int s = 1; s < a.splits; ++s) v += pb[(long)s * a.split_stride + i];
    row[i] = v;
    if (i < qd) ssq += v * v;
    else if (i < qd + kd) ssk += v * v;
  }
  if (a.q_norm_w) {
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
// row. Sub-groups of HD/8 lanes each own one position at a time and load its
// K and V rows with 16-byte vector loads; scores are reduced with warp
// shuffles and accumulated with an online softmax. Chunk boundaries are fixed
// multiples of kAttnChunk and positions map to warps by index, so results do
// not depend on the batch. Output: unnormalised partial (acc, max, sum) per
// chunk, merged by attn_combine_kernel in chunk order.
constexpr int kAttnChunk = 256;
constexpr int kAttnThreads = 128;
constexpr int kAttnUnroll = 4;

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
  float scale;
  int* err;
};

template <int HD, int G>
__global__ void __launch_bounds__(kAttnThreads) attn_kernel(AttnArgs a) {
  pdl_wait();
  pdl_launch_dependents();
  constexpr int LPP = HD / 8;          // lanes per position
  constexpr int PPW = 32 / LPP;        // positions per warp step
  constexpr int NW = kAttnThreads / 32;
  constexpr int STEP = NW * PPW;
  const int b = blockIdx.x, g = blockIdx.y, c = blockIdx.z;
  const int T = a.meta.get(kMetaPos, b) + 1;
  const int start = c * kAttnChunk;
  if (start >= T) return;
  const int end = min(start + kAttnChunk, T);
  const int row = a.meta.get(kMetaRow, b);
  if (row < 0 || row >= a.rows || T > a.max_ctx) {
    if (threadIdx.x == 0) atomicExch(a.err, kDevBadIndex);
    return;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sub = lane / LPP, sl = lane % LPP;
  const int kd = a.nkv * HD;
  const int* mrow = a.map + (long)row * a.max_ctx;

  float qv[G][8];
#pragma unroll
  for (int h = 0; h < G; ++h) {
    const float* qp = a.q + (long)b * a.nh * HD + (g * G + h) * HD + sl * 8;
#pragma unroll
    for (int d = 0; d < 8; ++d) qv[h][d] = qp[d] * a.scale;
  }
  float m[G], l[G], acc[G][8];
#pragma unroll
  for (int h = 0; h < G; ++h) {
    m[h] = -INFINITY;
    l[h] = 0.f;
#pragma unroll
    for (int d = 0; d < 8; ++d) acc[h][d] = 0.f;
  }

  // The loop bound is warp-uniform (jb is the same for every lane of a warp),
  // so all 32 lanes reach every shuffle below; out-of-range positions are
  // masked through `valid`.
  for (int jb = start + warp * PPW; jb < end; jb += STEP * kAttnUnroll) {
    uint4 kr[kAttnUnroll], vr[kAttnUnroll];
    bool valid[kAttnUnroll];
#pragma unroll
    for (int u = 0; u < kAttnUnroll; ++u) {
      const int j = jb + sub + u * STEP;
      int slot = j < end ? mrow[j] : -1;
      valid[u] = slot >= 0 && slot < a.n_slots;
      if (j < end && !valid[u]) atomicExch(a.err, kDevBadIndex);
      if (valid[u]) {
        const long off = (long)slot * kd + g * HD + sl * 8;
        kr[u] = *reinterpret_cast<const uint4*>(a.kpool + off);
        vr[u] = *reinterpret_cast<const uint4*>(a.vpool + off);
      }
    }
#pragma unroll
    for (int u = 0; u < kAttnUnroll; ++u) {
      float kf[8], vf[8];
      if (valid[u]) {
        unpack8(kr[u], kf);
        unpack8(vr[u], vf);
      }
#pragma unroll
      for (int h = 0; h < G; ++h) {
        float s = 0.f;
#pragma unroll
        for (int d = 0; d < 8; ++d) s += qv[h][d] * (valid[u] ? kf[d] : 0.f);
#pragma unroll
        for (int o = LPP / 2; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (valid[u]) {
          const float mn = fmaxf(m[h], s);
          const float corr = __expf(m[h] - mn);
          const float p = __expf(s - mn);
          l[h] = l[h] * corr + p;
#pragma unroll
          for (int d = 0; d < 8; ++d) acc[h][d] = acc[h][d] * corr + p * vf[d];
          m[h] = mn;
        }
      }
    }
  }

  // Merge sub-groups within the warp, then warps through shared memory.
  __shared__ float sm_m[NW][G], sm_l[NW][G];
  __shared__ float sm_acc[NW][G][HD];
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
}

// x[b][h*HD + d] = bf16(sum_c acc_c e^(m_c - M) / sum_c l_c e^(m_c - M)), chunks in order.
__global__ void attn_combine_kernel(Meta meta, int nh, int hd, int max_chunks,
                                    const float* __restrict__ o_part,
                                    const float* __restrict__ ml_part,
                                    __nv_bfloat16* __restrict__ x) {
  pdl_wait();
  pdl_launch_dependents();
  const int b = blockIdx.x, h = blockIdx.y;
  const int T = meta.get(kMetaPos, b) + 1;
  int nch = (T + kAttnChunk - 1) / kAttnChunk;
  if (nch > max_chunks) nch = max_chunks;
  const long base = ((long)b * nh + h) * max_chunks;
  float mm = -INFINITY;
  for (int c = 0; c < nch; ++c) mm = fmaxf(mm, ml_part[(base + c) * 2]);
  for (int d = threadIdx.x; d < hd; d += blockDim.x) {
    float ll = 0.f, aa = 0.f;
    for (int c = 0; c < nch; ++c) {
      const float w = mm == -INFINITY ? 0.f : __expf(ml_part[(base + c) * 2] - mm);
      ll += ml_part[(base + c) * 2 + 1] * w;
      aa += o_part[(base + c) * hd + d] * w;
    }
    store_pair(x, (long)nh * hd, b, h * hd + d, ll > 0.f ? aa / ll : 0.f);
  }
}

// ------------------------------------------------------------------ argmax
// out[b] = argmax_v logits[b][v], lowest index among equal maxima
// (torch.argmax semantics, sglang_recurrent/loopspec/decisions.py:116).
__global__ void argmax_kernel(const float* __restrict__ logits, int V, long ld,
                              long long* __restrict__ out) {
  pdl_wait();
  pdl_launch_dependents();
  const int b = blockIdx.x;
  const float* r = logits + (long)b * ld;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int v = threadIdx.x; v < V; v += blockDim.x) {
    const float x = r[v];
    if (x > best || (x == best && v < bi)) {
      best = x;
      bi = v;
    }
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
// Philox4x32-10 (Salmon, Moraes, Dror, Shaw, SC'11), counter = (i/4, pos, 0, 0).
__device__ __forceinline__ uint4 philox4x32_10(uint4 c, uint32_t k0, uint32_t k1) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t lo0 = 0xD2511F53u * c.x, hi0 = __umulhi(0xD2511F53u, c.x);
    const uint32_t lo1 = 0xCD9E8D57u * c.z, hi1 = __umulhi(0xCD9E8D57u, c.z);
    c = make_uint4(hi1 ^ c.y ^ k0, lo1, hi0 ^ c.w ^ k1, lo0);
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return c;
}

// bank_h[state_out] = truncnormal(0, std; +-3 std)(seed, pos) * scale;
// bank_inj[state_out] = h[b] (the prelude output).
__global__ void raven_init_kernel(Meta meta, int H, const float* __restrict__ h,
                                  float* __restrict__ bank_h, float* __restrict__ bank_inj,
                                  int bank_rows, unsigned long long seed, float std_,
                                  float scale, int* err) {
  pdl_wait();
  pdl_launch_dependents();
  const int b = blockIdx.x;
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
