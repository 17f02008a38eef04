// Host-visible part of the persistent stack kernel: the phase program format,
// the launch parameters and the entry points implemented in stack.cu. The
// device code is in stack.cuh.
#pragma once

#include "common.cuh"

namespace ls {

constexpr int kStkThreads = 288;         // warps 0 weights TMA, 1 MMA, 2..7 workers, 8 activation TMA
constexpr int kStkWorkers = 192;       // warps 2..7
constexpr int kStkWorkerTid0 = 64;
constexpr int kStkEpiTid0 = 128;       // warps 4..7 read TMEM
constexpr int kStkChunk = 96;          // attention positions per work item
constexpr int kStkRowNV = 8;           // float4 columns per worker per row: H <= 6144
constexpr int kStkMaxLanes = 128;
constexpr int kBarWorkers = 1, kBarEpi = 2;   // named barrier ids (0 is __syncthreads)
constexpr unsigned long long kStkWaitNs = 2000000000ull;   // any single wait: 2 s
constexpr unsigned long long kStkStartNs = 1000000000ull;  // co-residency check: 1 s

constexpr int kStkTraceFields = 12;

enum StkError : int { kDevTimeoutGrid = 5, kDevNotResident = 6 };

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

struct Phase {
  int kind;
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
  float* part_ws;                 // [grid][2][BN/2][128] segment partials
  int* tile_tickets;              // per-tile contributor counters, zero between phases
  unsigned* sync;                 // [0] start, [1] phase arrivals, [2] exits
  int* err;
  // optional timing trace, [n_phases + 1][grid][kStkTraceFields] globaltimer
  // ns, per phase: 0 start of work, 1 arrival, 2 first accumulator ready,
  // 3 first activation load issued, 4 work done, 5 fences done, 6 producer
  // saw the phase's inputs complete, 7 last segment finished, 8 last
  // activation load issued, 9 MMA took its first stage, 10 MMA finished its
  // first segment, 11 weight stages of the phase already issued when its
  // inputs were seen complete (a count); row n_phases: kernel entry (0) and
  // co-residency pass (1).
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

constexpr int stk_stages(int bn) { return bn <= 16 ? 11 : bn <= 32 ? 10 : bn <= 64 ? 8 : bn <= 128 ? 6 : 4; }
cudaError_t stack_prepare();
cudaError_t stack_launch(int bn, int hd, const StackLaunch& L, int grid, cudaStream_t stream, bool pdl);
size_t stack_smem_bytes(int bn);

}  // namespace ls
