// Host-visible part of the persistent stack kernel: the phase program format,
// the launch parameters and the entry points implemented in stack.cu. The
// device code is in stack.cuh.
#pragma once

#include "common.cuh"

namespace ls {

constexpr int kStkThreads = 288;         // warps 0 weights TMA, 1 MMA, 2 activation TMA, 3..8 workers
constexpr int kStkWorkers = 192;       // warps 3..8
constexpr int kStkWorkerTid0 = 96;
static_assert(kStkWorkerTid0 <= 128 && 128 + 128 <= kStkWorkerTid0 + kStkWorkers,
              "the epilogue warps 4..7 must be workers");
constexpr int kStkEpiTid0 = 128;       // warps 4..7 (a subset of the workers) read TMEM
constexpr int kStkChunk = 96;          // attention positions per work item
constexpr int kStkRowNV = 8;           // float4 columns per worker per row: H <= 6144
constexpr int kStkMaxLanes = 128;
constexpr int kBarWorkers = 1, kBarEpi = 2;   // named barrier ids (0 is __syncthreads)
constexpr unsigned long long kStkWaitNs = 2000000000ull;   // any single wait: 2 s
constexpr unsigned kStkPollNs = 100;                        // back-off between counter polls
constexpr unsigned long long kStkStartNs = 1000000000ull;  // co-residency check: 1 s

constexpr int kStkTraceFields = 12;

enum StkError : int { kDevTimeoutGrid = 5, kDevNotResident = 6 };   // 5: a dependency wait timed out

enum PhaseKind : int {
  kPhMap = 0,      // timeline mapping: fork copy + append (map_update_kernel)
  kPhPrep = 1,     // h = embed or bank[state_in]; optional bank / x outputs
  kPhCat = 2,      // Raven adapter input (hi, lo) of [bank_h, bank_inj]
  kPhGemm = 3,     // weight GEMM with a store / RoPE+KV / SwiGLU epilogue
  kPhQkNorm = 4,   // OLMo2 QK-norm + RoPE + KV write from the stored QKV rows
  kPhAttn = 5,     // paged decode attention over the lanes' timelines
  kPhRow = 6,      // residual / norm row epilogue (resid_epi_kernel semantics)
  kPhRavenInit = 7 // Raven position-keyed hidden init (raven_init_kernel)
};

enum XBufId : int { kXH = 0, kXAttn = 1, kXAct = 2, kXCat = 3, kXBufs = 4 };

// Dependency kinds: what a phase's work waits for (counter >= target).
enum DepKind : int {
  kDepNone = 0,
  kDepTotLanes = 1,   // tot[q] >= lanes of the call (a per-lane phase finished)
  kDepTotTiles = 2,   // tot[q] >= tiles of GEMM phase q (all its tiles stored)
  kDepKbHead = 3,     // GEMM activation k-block kb: cnt[q][kv head of kb] >= lanes (attention q)
  kDepKbTile = 4,     // GEMM activation k-block kb: cnt[q][kb] >= 1 (tile kb of GEMM q)
  kDepQkvHead = 5,    // attention item of kv head g: the QKV tiles holding g's q, k, v rows
};

struct Phase {
  int kind;
  int cnt_off;                               // this phase's per-tile / per-head counters, or -1
  int gemm_idx;                              // ordinal among the program's GEMM phases
  int dep_kind[2], dep_phase[2];             // inputs this phase's work waits for
  // GEMM
  int xbuf, epi, Mw, K, m_tiles, KB, head;   // head: lanes [head_lane0, +head_n)
  int wmap;                                  // index into StackLaunch::wmap
  float* out;                                // store epilogue: out[lane][Mw]
  // this layer's KV pools (QKV epilogue, QK-norm, attention)
  __nv_bfloat16* kpool;
  __nv_bfloat16* vpool;
  // rows (kPhRow / kPhPrep)
  const float* src;                          // row: GEMM output; prep: bank (null: embedding)
  const __nv_bfloat16* bias;
  const __nv_bfloat16* a_norm_w;
  const float* resid;
  float* out_h;
  const __nv_bfloat16* final_norm_w;
  float* bank;                               // also write the row to bank[state_out]
  int x_out;                                 // -1 or the x buffer receiving (hi, lo)
  const __nv_bfloat16* x_norm_w;
  const __nv_bfloat16* q_norm_w;             // QK-norm
  const __nv_bfloat16* k_norm_w;
};

struct StackParams {
  const Phase* phases;
  int n_phases;
  Meta meta;
  int n;                          // lanes of the call
  int head_lane0, head_n;         // lanes of head GEMMs
  __nv_bfloat16* x[kXBufs];
  int xK[kXBufs];
  float* h;
  float* q;
  int H, NH, NKV, HD, I;
  const float* inv_freq;
  float eps, attn_scale;
  const __nv_bfloat16* embed;
  float embed_scale;
  int vocab;
  int* map;
  int max_ctx, rows, n_slots;
  float* bank_h;
  float* bank_inj;
  int bank_rows;
  unsigned long long init_seed;
  float init_std;
  float* o_part;                  // [cap][NH][max_chunks][HD]
  float* ml_part;                 // [cap][NH][max_chunks][2]
  int* attn_tickets;              // [cap][NKV]
  int max_chunks;
  float* part_ws;                 // [2][grid][2][BN/2][128] segment partials (GEMM parity)
  int* tile_tickets;              // [2][max tiles] contributor counters, zero between uses
  int* cnt;                       // completion counters: per tile / per head, zero between launches
  int* tot;                       // [n_phases] per-phase completion counters
  int n_cnt;                      // entries of cnt (reset at exit)
  int ticket_stride;              // tile tickets per GEMM parity
  unsigned* sync;                 // [0] start, [2] exits
  int* err;
  // optional timing trace, [n_phases + 1][grid][kStkTraceFields] globaltimer
  // ns, per phase and CTA: 0 start of work, 1 end of work, 2 first
  // accumulator ready, 3 first activation load issued, 6 inputs of the first
  // activation load seen complete, 8 last activation load issued, 9 MMA took
  // its first stage, 10 MMA finished its first segment, 11 weight stages of
  // the phase already issued when its inputs were seen (a count); row
  // n_phases: kernel entry (0) and co-residency pass (1).
  unsigned long long* trace;
};

// Host entry points (stack.cu): stages per BN keep the ring near 200 KB.
// Kernel parameter block: the tensor maps live in parameter space (the TMA
// unit reads them through the constant cache), up to kStkMaxMaps weight maps
// per program; 26.5 KB, under the 32 KB kernel-parameter limit.
constexpr int kStkMaxMaps = 200;
struct StackLaunch {
  CUtensorMap xmap[kXBufs];       // activation maps with BN-row boxes
  CUtensorMap wmap[kStkMaxMaps];  // weight maps, indexed by Phase::wmap
  StackParams P;
};
static_assert(sizeof(StackLaunch) <= 32764, "kernel parameters above the 32 KB limit");

// A ring stage holds one k-unit of kStkBK = 128: two 64-wide (128-byte
// swizzle) sub-tiles per operand, so the MMA issuer's per-stage overhead
// (commit, barrier wait, loop) is paid once per 32 KB of weights.
constexpr int kStkBK = 128;
constexpr int kStkSub = kStkBK / 64;
constexpr int stk_stages(int bn) { return bn <= 32 ? 5 : bn <= 64 ? 4 : bn <= 128 ? 3 : 2; }
cudaError_t stack_prepare();
cudaError_t stack_launch(int bn, int hd, const StackLaunch& L, int grid, cudaStream_t stream, bool pdl);
size_t stack_smem_bytes(int bn);

}  // namespace ls
