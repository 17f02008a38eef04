// LoopSpec decode engine for B200 (sm_100a): host runtime and C ABI.
//
// The engine owns, per model: the paged KV pool (one slot per token per
// timeline, page size 1), the timeline mapping table (row -> slot per
// position), the hidden/injected state banks, and the workspaces of one role
// call. A role call (pre / core / post over B lanes) is a fixed kernel
// sequence that reads lane metadata from a device buffer, so it is captured
// once per (role, B) as a CUDA graph and replayed after a small metadata
// upload. The host side restates the reference's branch-timeline bookkeeping
// (sglang_recurrent/loopspec/branching/manager.py), executor
// (loopspec/executor.py) and scheduler loop (loopspec/pipeline.py) in C++ so a
// whole request runs without Python in the loop.

#include "../../include/loopspec_engine.h"
#include "common.cuh"
#include "dev_sched.cuh"
#include "gemm_tc.cuh"
#include "kernels.cuh"
#include "prefill_attn.cuh"
#include "sampler.cuh"

#include <algorithm>
#include <array>
#include <chrono>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <map>
#include <memory>
#include <mutex>
#include <queue>
#include <set>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

using namespace ls;
typedef __nv_bfloat16 bf16;

namespace {

struct EngineError : std::runtime_error {
  int code;
  EngineError(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

// Error text of the last failed call that has no engine handle.
thread_local std::string g_last_error;

#define CK(x)                                                                            \
  do {                                                                                   \
    cudaError_t e_ = (x);                                                                \
    if (e_ != cudaSuccess)                                                               \
      throw EngineError(LS_ECUDA, std::string(#x) + ": " + cudaGetErrorString(e_));      \
  } while (0)

#define REQUIRE(cond, code, msg)                  \
  do {                                                \
    if (!(cond)) throw EngineError((code), (msg));    \
  } while (0)

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    CK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
    REQUIRE(q == cudaDriverEntryPointSuccess && p, LS_ECUDA, "cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 2-D bf16 tensor map [rows][inner], 128-byte swizzle, box {64, box_rows}.
CUtensorMap make_map_2d(const void* base, uint64_t inner, uint64_t rows, uint32_t box_rows) {
  REQUIRE((reinterpret_cast<uintptr_t>(base) & 15) == 0, LS_EINVAL, "TMA base must be 16-byte aligned");
  REQUIRE((inner * 2) % 16 == 0, LS_EINVAL, "TMA row pitch must be a multiple of 16 bytes");
  CUtensorMap m;
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {inner * 2};
  cuuint32_t box[2] = {(cuuint32_t)kGemmBK, box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = get_encode()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                            strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  REQUIRE(r == CUDA_SUCCESS, LS_ECUDA, "cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
  return m;
}

int round_up(int x, int m) { return (x + m - 1) / m * m; }
int cdiv(long a, long b) { return (int)((a + b - 1) / b); }

struct Gemm {
  const bf16* w = nullptr;
  int Mw = 0, K = 0, splits = 1;
  CUtensorMap map;      // 128-row weight boxes
  CUtensorMap map64;    // 64-row boxes (gate/up halves of the SwiGLU tile)
  bool has_map64 = false;
  bool cluster = false;  // split store: the tile's splits add their partials in the GEMM (one plane)
};

struct XBuf {
  bf16* ptr = nullptr;
  int K = 0, rows = 0;
  std::map<int, CUtensorMap> by_bn;
  const CUtensorMap& map(int bn) {
    auto it = by_bn.find(bn);
    if (it == by_bn.end()) it = by_bn.emplace(bn, make_map_2d(ptr, K, rows, bn)).first;
    return it->second;
  }
};

struct LayerW {
  const bf16 *qkv = nullptr, *o = nullptr, *gu = nullptr, *down = nullptr;
  const bf16 *n_in = nullptr, *n_pa = nullptr, *n_pf = nullptr, *n_pff = nullptr;
  const bf16 *qn = nullptr, *kn = nullptr;
  Gemm g_qkv, g_o, g_gu, g_down;
};

enum Role { kPre = 0, kCore = 1, kPost = 2 };

struct Stack {
  std::vector<LayerW> layers;
  int kv_base = 0;
};

// What the last layer of a stack produces besides h.
struct StackEnd {
  const bf16* final_norm = nullptr;  // Ouro step_norm
  float* bank = nullptr;             // scatter h into this bank at state_out
  bool want_x = false;               // produce x for a following GEMM
  const bf16* x_norm = nullptr;      // ... normalised by this weight (Raven ln_f)
};

// Launch with optional programmatic-dependent-launch attribute.
template <typename... KArgs, typename... Args>
void launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl,
            Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = pdl ? attr : nullptr;
  cfg.numAttrs = pdl ? 1 : 0;
  CK(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...));
}

double now_s() {
  return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

}  // namespace

// ===================================================================== timelines
// Host bookkeeping of branch KV timelines, restating
// sglang_recurrent/loopspec/branching/manager.py:
//   TimelineCursor :45-63, _TimelineManager.fork :207-232 / release :234-250,
//   BranchManager.get_or_create_cursors :357-388, _release_unused_branch
//   :390-408, _transfer_timeline_ownership :410-429, _detach_from_unused_parent
//   :431-451, retain_branches :453-482.
// Rows index the device mapping table; slots index the KV pool. Both come from
// free stacks owned here (the reference keeps a GPU-side slot ring mirrored on
// the CPU, decode_slots.py; this engine uploads the chosen slot ids with the
// lane metadata instead).
namespace {

struct Cursor {
  int row = -1;
  int seq_len = 0;
  int pending_parent_row = -1;
  std::vector<int> owned;   // decode slots this cursor frees on release
};

struct Node {
  int id = 0;
  Node* parent = nullptr;
  std::map<int, Cursor*> cur[3];
  int child_count = 0;
  bool live = true;
};

class Timelines {
 public:
  // A request owns mapping rows [row_base, row_base + rows) and KV slots
  // [slot_base, slot_base + slots); requests batched in one engine get
  // disjoint ranges.
  void configure(int rows, int slots, int row_base = 0, int slot_base = 0) {
    rows_ = rows;
    slots_ = slots;
    row_base_ = row_base;
    slot_base_ = slot_base;
    reset();
  }

  void reset() {
    for (auto& kv : nodes_) {
      for (auto& m : kv.second->cur)
        for (auto& c : m) delete c.second;
      delete kv.second;
    }
    nodes_.clear();
    free_rows_.clear();
    for (int r = rows_ - 1; r >= 0; --r) free_rows_.push_back(row_base_ + r);
    free_slots_.clear();
    for (int s = slots_ - 1; s >= 0; --s) free_slots_.push_back(slot_base_ + s);
  }

  ~Timelines() { reset(); }

  int alloc_slot() {
    REQUIRE(!free_slots_.empty(), LS_ECAPACITY, "KV slot pool exhausted");
    int s = free_slots_.back();
    free_slots_.pop_back();
    return s;
  }

  int alloc_row() {
    REQUIRE(!free_rows_.empty(), LS_ECAPACITY, "recurrent branch ran out of request-pool rows");
    int r = free_rows_.back();
    free_rows_.pop_back();
    return r;
  }

  // A full-prompt timeline owned by the root; its prompt slots are returned
  // with the whole pool at request end, as the reference's eager prefill does.
  Cursor* create_root_cursor(int role, int depth) {
    Node* root = node_or_null(0);
    if (!root) {
      root = new Node();
      nodes_[0] = root;
    }
    Cursor* c = new Cursor();
    c->row = alloc_row();
    root->cur[role][depth] = c;
    return c;
  }

  Node* node_or_null(int id) {
    auto it = nodes_.find(id);
    return it == nodes_.end() ? nullptr : it->second;
  }

  Node* get_or_create_branch(int id, int parent_id) {
    Node* n = node_or_null(id);
    if (n) return n;
    Node* p = node_or_null(parent_id);
    REQUIRE(p, LS_EPIPELINE,
            "branch " + std::to_string(id) + " has unavailable parent " + std::to_string(parent_id));
    n = new Node();
    n->id = id;
    n->parent = p;
    p->child_count += 1;
    nodes_[id] = n;
    return n;
  }

  Cursor* get_or_create_cursor(int role, int depth, int branch, int parent) {
    Node* n = get_or_create_branch(branch, parent);
    auto it = n->cur[role].find(depth);
    if (it != n->cur[role].end()) return it->second;
    REQUIRE(n->parent, LS_EPIPELINE, "root branch is missing a timeline");
    auto pit = n->parent->cur[role].find(depth);
    REQUIRE(pit != n->parent->cur[role].end(), LS_EPIPELINE, "parent timeline missing for fork");
    Cursor* c = new Cursor();
    c->row = alloc_row();
    c->seq_len = pit->second->seq_len;
    c->pending_parent_row = pit->second->row;
    n->cur[role][depth] = c;
    return c;
  }

  void retain(const std::vector<std::pair<int, int>>& lanes /* (branch, parent) */) {
    std::vector<std::pair<int, int>> sorted = lanes;
    std::sort(sorted.begin(), sorted.end());
    for (auto& bp : sorted)
      if (bp.first && !node_or_null(bp.first)) get_or_create_branch(bp.first, bp.second);
    std::set<int> keep;
    for (auto& bp : lanes) keep.insert(bp.first);
    std::vector<int> unused;
    for (auto& kv : nodes_)
      if (kv.second->live && !keep.count(kv.first)) unused.push_back(kv.first);
    std::sort(unused.rbegin(), unused.rend());
    for (int id : unused) {
      Node* n = node_or_null(id);
      if (!n) continue;
      n->live = false;
      release_unused(n);
    }
    std::vector<int> ids;
    for (auto& kv : nodes_) ids.push_back(kv.first);
    for (int id : ids) {
      Node* n = node_or_null(id);
      if (n) detach_from_unused_parent(n);
    }
  }

  size_t live_nodes() const { return nodes_.size(); }

  // Hand a freshly prefilled request to the device loop's scheduler `d`
  // (whose root node is d.nodes[0]): the root's cursors, the free mapping
  // rows, and the free KV slots, which after a prefill are one contiguous
  // range [first free, slot_base + slots).
  template <class D>
  void export_to(D& d) const {
    auto it = nodes_.find(0);
    REQUIRE(it != nodes_.end() && nodes_.size() == 1, LS_EINVAL, "device loop needs a freshly prefilled request");
    for (int role = 0; role < 3; ++role)
      for (auto& kv : it->second->cur[role]) {
        REQUIRE(kv.first < (int)(sizeof(d.kind_of) / sizeof(int)), LS_EINVAL, "timeline depth beyond the device loop");
        d.nodes[0].cur[role][kv.first] = d.new_cursor(kv.second->row, kv.second->seq_len, -1);
      }
    REQUIRE(free_rows_.size() <= sizeof(d.free_rows) / sizeof(int), LS_ECAPACITY, "too many rows for the device loop");
    d.n_free_rows = (int)free_rows_.size();
    for (size_t i = 0; i < free_rows_.size(); ++i) d.free_rows[i] = free_rows_[i];
    REQUIRE(!free_slots_.empty(), LS_ECAPACITY, "KV slot pool exhausted");
    const int first = free_slots_.back();
    REQUIRE((int)free_slots_.size() == slot_base_ + slots_ - first, LS_EINVAL, "free KV slots are not contiguous");
    d.next_slot = first;
    d.slot_limit = slot_base_ + slots_;
  }
  size_t free_slots() const { return free_slots_.size(); }
  size_t free_rows() const { return free_rows_.size(); }

 private:
  void release_cursor(Cursor* c) {
    for (int s : c->owned) free_slots_.push_back(s);
    free_rows_.push_back(c->row);
    delete c;
  }

  void release_unused(Node* n) {
    while (n && !n->live && n->child_count == 0) {
      for (auto& m : n->cur)
        for (auto& c : m) release_cursor(c.second);
      Node* p = n->parent;
      nodes_.erase(n->id);
      delete n;
      if (!p) break;
      p->child_count -= 1;
      n = p;
    }
  }

  void detach_from_unused_parent(Node* n) {
    Node* p = n->parent;
    if (!p || p->live || p->child_count != 1) return;
    for (int role = 0; role < 3; ++role) {
      auto& pc = p->cur[role];
      auto& cc = n->cur[role];
      for (auto it = pc.begin(); it != pc.end();) {
        auto cit = cc.find(it->first);
        if (cit == cc.end()) {
          cc[it->first] = it->second;
          it = pc.erase(it);
        } else {
          auto& own = cit->second->owned;
          own.insert(own.begin(), it->second->owned.begin(), it->second->owned.end());
          it->second->owned.clear();
          ++it;
        }
      }
    }
    n->parent = nullptr;
    p->child_count -= 1;
    release_unused(p);
  }

  int rows_ = 0, slots_ = 0, row_base_ = 0, slot_base_ = 0;
  std::map<int, Node*> nodes_;
  std::vector<int> free_rows_, free_slots_;
};

}  // namespace

namespace {
// One request of a batch: its branch timelines (disjoint mapping rows and KV
// slots), prompt length, random-stream cycle counter and sampling seed. Its
// recurrent state slots are [state_base, state_base + max_rows).
struct Request {
  Timelines tl;
  int prefill_len = -1;     // len(prompt) - 1
  uint32_t draw_cycle = 0;  // the first token uses draw 0, decode cycles 1, 2, ...
  unsigned long long seed = 0;
  int state_base = 0;
  bool sampled = false;     // top-p / top-k / temperature decisions (else greedy)
};
}  // namespace

namespace {
// Sampling parameters as the engine stores them: greedy iff top_k == 1
// (temperature 0 is normalised to it), as the reference server decides
// (server/loopspec_scheduler.py:316-329).
SampleParams sample_params(float temperature, int top_k, float top_p, unsigned long long seed) {
  const bool greedy = temperature == 0.f || top_k == 1;
  return SampleParams{temperature == 0.f ? 1.f : temperature, top_p, greedy ? 1 : top_k, 0, seed};
}
bool params_sampled(const SampleParams& p) { return p.top_k != 1; }
}  // namespace

// ======================================================================= engine
struct ls_engine {
  ls_model_cfg mc{};
  ls_sched_cfg sc{};
  int device = 0;
  int num_sms = 148;
  std::string last_error;
  bool finalized = false;

  // schedule (pipeline.py:124-251)
  int S = 0, K = 1, X = 0;
  std::map<int, int> endpoint_kind;  // end stage -> 0 q1, 1 q2, 2 final
  int max_rows = 0, depth = 0;

  // weights
  std::map<std::string, std::pair<const bf16*, std::vector<int64_t>>> weights;
  Stack pre, core, post;
  const bf16 *embed = nullptr, *lm_head = nullptr, *step_norm = nullptr, *final_norm = nullptr;
  const bf16 *adapter_b = nullptr;
  Gemm g_adapter, g_lm;

  // sizes
  int H = 0, QD = 0, KVD = 0, I = 0, V = 0, HD = 0, NH = 0, NKV = 0;
  int cap = 0;           // lanes per role call
  int prefill_chunk = 128;
  int n_attn_layers = 0, n_slots = 0, rows = 0, max_ctx = 0, max_chunks = 0, bank_rows = 0;

  // device memory
  cudaStream_t stream = nullptr;
  std::vector<void*> allocs;
  bf16 *kpool = nullptr, *vpool = nullptr;
  int* map = nullptr;
  float *bank_h = nullptr, *bank_inj = nullptr;
  int* meta_dev = nullptr;      // [3][F][cap]
  const int* meta_override = nullptr;   // metadata of the role call being enqueued, if not meta_dev's
  // device-resident decode loop (greedy, one request): the scheduler state,
  // the metadata of one cycle's role calls ([pre][K core][post], width
  // max_rows), committed tokens, and the captured cycle graph
  LoopSched* loop_sched = nullptr;
  LoopSched* loop_host = nullptr;   // pinned
  int* loop_meta = nullptr;
  long long* loop_out = nullptr;
  struct LoopGraph {
    cudaGraphExec_t exec = nullptr;
    int kernels = 0;
  };
  // one cycle's graph per (attention chunks, sampling): key chunks * 2 + sampling
  std::map<int, LoopGraph> loop_graphs;
  int attn_form_lanes = 0;   // lanes assumed by the attention form choice (0: the call's width)
  int* loop_active = nullptr;       // live lanes of the device loop's pre, core, post calls
  const int* gemm_active = nullptr;  // set while the device loop's calls are captured
  int* meta_host = nullptr;     // pinned [kStaging][F][cap]
  int staging_next = 0;
  static constexpr int kStaging = 64;
  float *h = nullptr, *r = nullptr, *q = nullptr, *part = nullptr, *o_part = nullptr,
        *ml_part = nullptr, *logits = nullptr, *inv_freq = nullptr;
  long part_elems = 0;
  XBuf x_h, x_attn, x_act, x_cat;
  long long *amax_dev = nullptr, *amax_host = nullptr;
  // greedy tokens fused into the lm_head GEMM: per-lane tile maxima and the
  // grid's arrival counter (zero between launches)
  float* amax_val = nullptr;
  int *amax_idx = nullptr, *amax_ticket = nullptr;
  float* logits_host = nullptr;
  int* err_dev = nullptr;
  int* err_host = nullptr;      // pinned copy of err_dev, fetched with each step's results
  int* attn_tickets = nullptr;  // [cap][n_kv_heads] chunk-arrival counters, zero between calls
  // sampling (greedy iff disabled): parameters on the device so captured
  // graphs read the current request's settings; q1 / q2-residual
  // distributions per lane state slot; per-row scratch and decisions
  bool sampling = false;
  SampleParams sparams{1.f, 1.f, 0, 0, 0ull};
  SampleParams* sparams_dev = nullptr;
  float *q1_bank = nullptr, *r_bank = nullptr;
  long long *dec_dev = nullptr, *dec_host = nullptr;
  float* gemm_part = nullptr;   // GEMM split partial tiles
  long gemm_part_elems = 0;
  int* gemm_tickets = nullptr;  // GEMM per-tile split-arrival counters, zero between launches
  long gemm_ticket_count = 0;
  cudaEvent_t ev0 = nullptr, ev1 = nullptr;

  std::map<std::pair<int, int>, cudaGraphExec_t> graphs;
  std::map<std::pair<int, int>, int> graph_kernels;   // kernels per captured graph
  std::map<std::pair<int, int>, int> graph_chunks;    // attention grid chunks per graph
  std::map<std::pair<int, int>, bool> graph_planes;   // decode-form QKV per graph
  // Decode form of the call being enqueued: every lane has one new position,
  // so the QKV projection stores split planes and attention finishes q / K / V
  // (RoPE, pool write) itself. Prefill calls (several positions of one
  // timeline) keep the projection's fused RoPE / KV-write epilogue.
  bool qkv_planes = false;
  // attention grid depth of the call being enqueued: one CTA per 128-position
  // chunk of its longest timeline (graphs round it up to an even count and are
  // re-captured when it changes)
  int attn_chunks = 1;
  int64_t kernel_launches = 0;                        // kernels launched by role calls
  // work counters of role calls (decode stats are differences around the loop)
  int64_t pre_calls = 0, core_calls = 0, core_kv_positions = 0, post_calls = 0;
  int64_t host_syncs = 0;   // stream synchronisations of decode loops
  int kernels_in_call = 0;
  // The next launch waits for full completion of the previous kernel (no
  // programmatic overlap). Set after the mapping update: every kernel
  // triggers its dependents at its start, and attention reads the
  // timeline's slot ids before its own wait.
  bool serialize_next = false;
  int meta_after_wait = 0;   // the next prep kernel reads its metadata only after its PDL wait
  // Set while prefill runs: its calls are up to 128 lanes wide, where the
  // QKV and gate_up projections are compute-bound, so they run unsplit (the
  // epilogue then reads the tile from shared memory instead of re-reading
  // every split's partial tile from global memory). Decode calls keep the
  // fixed splits; both generation modes share the same prefill.
  bool prefill_mode = false;
  int64_t h2d_bytes = 0, d2h_bytes = 0;   // host<->device traffic counters

  // Tensor parallelism (ls_tp_init / ls_tp_attach): this rank's exchange
  // region, one allocation so that one IPC handle maps it: flags and epoch
  // (first 256 bytes), the O and down projections' split planes, the QK-norm
  // sums. tp_base holds every rank's region in rank order (this rank's own
  // included); the layers exchange only once tp_ranks > 1 (after attach).
  int tp_ranks = 1, tp_rank = 0, tp_want = 1;
  char* tp_region = nullptr;
  size_t tp_bytes = 0, tp_off_o = 0, tp_off_d = 0, tp_off_qk = 0;
  std::vector<char*> tp_base;
  std::vector<void*> tp_opened;   // peer mappings, closed before the engine frees memory
  unsigned long long tp_wait_ns = kTpWaitNs;

  // Requests served together (ls_generate_batch); single-request entry points
  // use reqs[0]. max_state = max_req * max_rows state slots in the banks.
  std::vector<Request> reqs;
  int max_req = 1, max_state = 0;

  // ----------------------------------------------------------------- memory
  template <typename T>
  T* dalloc(size_t n) {
    void* p = nullptr;
    CK(cudaMalloc(&p, std::max<size_t>(n, 1) * sizeof(T)));
    CK(cudaMemset(p, 0, std::max<size_t>(n, 1) * sizeof(T)));
    allocs.push_back(p);
    return static_cast<T*>(p);
  }

  ~ls_engine() {
    if (device >= 0) cudaSetDevice(device);
    for (auto& g : graphs) cudaGraphExecDestroy(g.second);
    for (auto& g : loop_graphs) cudaGraphExecDestroy(g.second.exec);
    if (loop_host) cudaFreeHost(loop_host);
    for (void* p : tp_opened) cudaIpcCloseMemHandle(p);
    for (void* p : allocs) cudaFree(p);
    if (meta_host) cudaFreeHost(meta_host);
    if (amax_host) cudaFreeHost(amax_host);
    if (logits_host) cudaFreeHost(logits_host);
    if (dec_host) cudaFreeHost(dec_host);
    if (err_host) cudaFreeHost(err_host);
    if (ev0) cudaEventDestroy(ev0);
    if (ev1) cudaEventDestroy(ev1);
    if (stream) cudaStreamDestroy(stream);
  }

  // ---------------------------------------------------------------- weights
  const bf16* W(const std::string& name, std::vector<int64_t> shape, bool required = true) {
    auto it = weights.find(name);
    if (it == weights.end()) {
      REQUIRE(!required, LS_EINVAL, "missing weight " + name);
      return nullptr;
    }
    REQUIRE(it->second.second == shape, LS_EINVAL, "weight " + name + " has the wrong shape");
    return it->second.first;
  }

  // K splits per 128-row tile, aiming at about two CTAs per SM (all resident
  // in one wave), at most kMaxSplits. Measured on B200 (Ouro-1.4B core GEMMs,
  // 1-4 lanes): two per SM beats three or four per SM and beats 128-wide
  // stages, which halve the CTAs per SM. Depends only on the weight shape, never
  // on the batch.
  int choose_splits(int Mw, int Kd) const {
    const int tiles = cdiv(Mw, kGemmBM);
    const int KB = cdiv(Kd, kGemmBK);
    int s = (2 * num_sms + tiles / 2) / tiles;
    return std::max(1, std::min(std::min(s, KB), kMaxSplits));
  }

  Gemm cluster_gemm(const bf16* w, int Mw, int Kd) {
    Gemm g = make_gemm(w, Mw, Kd, std::min(choose_splits(Mw, Kd), kMaxClusterSplits));
    g.cluster = g.splits > 1;
    return g;
  }

  Gemm make_gemm(const bf16* w, int Mw, int Kd, int splits = 0, bool swiglu = false) {
    Gemm g;
    g.w = w;
    g.Mw = Mw;
    g.K = Kd;
    g.splits = splits > 0 ? splits : choose_splits(Mw, Kd);
    g.map = make_map_2d(w, Kd, Mw, kGemmBM);
    if (swiglu) {
      REQUIRE(Mw % kGemmBM == 0, LS_EINVAL, "gate_up rows must be a multiple of 128");
      g.map64 = make_map_2d(w, Kd, Mw, kGemmBM / 2);
      g.has_map64 = true;
    }
    part_elems = std::max(part_elems, (long)cap * Mw * g.splits);   // split planes
    // scratch for the widest call of this GEMM (cap lanes)
    const int bn = cap * 2 <= 16 ? 16 : cap * 2 <= 32 ? 32 : cap * 2 <= 64 ? 64 : cap * 2 <= 128 ? 128 : 256;
    const long tiles = (long)cdiv(Mw, kGemmBM) * cdiv(2 * cap, bn);
    gemm_ticket_count = std::max(gemm_ticket_count, tiles);
    if (g.splits > 1)
      gemm_part_elems = std::max(gemm_part_elems, tiles * g.splits * (bn / 2) * kGemmBM);
    return g;
  }

  void load_stack(Stack& st, const std::string& prefix, int n) {
    const int L = mc.layout;
    st.layers.resize(n);
    for (int i = 0; i < n; ++i) {
      const std::string p = prefix + std::to_string(i) + ".";
      LayerW& lw = st.layers[i];
      lw.qkv = W(p + "self_attn.qkv_proj.weight", {QD + 2 * KVD, H});
      lw.o = W(p + "self_attn.o_proj.weight", {H, QD});
      lw.gu = W(p + "mlp.gate_up_proj.weight", {2 * I, H});
      lw.down = W(p + "mlp.down_proj.weight", {H, I});
      if (L == LS_LAYOUT_OURO || L == LS_LAYOUT_RAVEN_PRE)
        lw.n_in = W(p + "input_layernorm.weight", {H});
      lw.n_pa = W(p + "post_attention_layernorm.weight", {H});
      if (L == LS_LAYOUT_OURO) lw.n_pf = W(p + "pre_feedforward_layernorm.weight", {H});
      if (L == LS_LAYOUT_OURO || L == LS_LAYOUT_OLMO_POST)
        lw.n_pff = W(p + "post_feedforward_layernorm.weight", {H});
      if (mc.qk_norm) {
        lw.qn = W(p + "self_attn.q_norm.weight", {QD});
        lw.kn = W(p + "self_attn.k_norm.weight", {KVD});
      }
      lw.g_qkv = make_gemm(lw.qkv, QD + 2 * KVD, H);
      // O and down (and the adapter): at most 16 K splits, added inside the
      // GEMM by each tile's cluster, so the row kernel after them reads one plane
      lw.g_o = cluster_gemm(lw.o, H, QD);
      lw.g_gu = make_gemm(lw.gu, 2 * I, H, 0, true);
      lw.g_down = cluster_gemm(lw.down, H, I);
    }
  }

  // The device-resident loop serves one greedy request of a schedule whose
  // lanes fit its fixed tables (at most 16 live lanes, S <= 8), on one GPU.
  bool loop_enabled = false;   // finalize sized the KV pool for the device loop
  bool device_loop_possible() const {
    return sc.device_loop && max_rows <= kLoopMaxLanes && S <= 8 && K <= kLoopMaxK && sc.use_graphs;
  }

  // ---------------------------------------------------------------- finalize
  void finalize() {
    REQUIRE(!finalized, LS_EINVAL, "engine already finalized");
    CK(cudaSetDevice(device));
    CK(cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, device));
    int major = 0, minor = 0;
    CK(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device));
    CK(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device));
    REQUIRE(major == 10 && minor == 0, LS_ECUDA, "this engine is built for sm_100a (B200) only");
    CK(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
    CK(cudaEventCreate(&ev0));
    CK(cudaEventCreate(&ev1));

    H = mc.hidden;
    NH = mc.n_heads;
    NKV = mc.n_kv_heads;
    HD = mc.head_dim;
    QD = NH * HD;
    KVD = NKV * HD;
    I = mc.intermediate;
    V = mc.vocab;
    REQUIRE(NH % NKV == 0, LS_EINVAL, "n_heads must be a multiple of n_kv_heads");
    const int G = NH / NKV;
    REQUIRE((HD == 64 && (G == 1 || G == 2 || G == 4)) || (HD == 128 && (G == 1 || G == 2)),
            LS_EINVAL, "unsupported head_dim / GQA group");
    REQUIRE(H % 64 == 0 && I % 64 == 0 && QD % 64 == 0, LS_EINVAL, "hidden/intermediate must be multiples of 64");
    REQUIRE(H % 128 == 0 && H <= 8192 && QD + 2 * KVD <= 12288, LS_EINVAL,
            "hidden must be a multiple of 128 and at most 8192 for the row kernels");

    max_req = std::max(1, sc.max_requests);
    REQUIRE(max_req <= 64, LS_EINVAL, "at most 64 requests per batch");
    max_state = max_req * max_rows;
    cap = std::max(max_state, prefill_chunk);
    max_ctx = sc.max_context;
    REQUIRE(max_ctx > 1 && sc.max_prompt >= 1 && sc.max_prompt < max_ctx, LS_EINVAL,
            "need 1 <= max_prompt < max_context");
    max_chunks = cdiv(max_ctx, kAttnChunk);
    REQUIRE(max_chunks <= kAttnMaxChunks, LS_EINVAL, "max_context above the attention kernel's limit");
    bank_rows = max_state + prefill_chunk;   // state slots, then prefill scratch rows
    n_attn_layers = mc.n_pre_layers + mc.n_core_layers + mc.n_post_layers;

    // timelines per branch: pre (if attention), S core, one post per endpoint
    const int n_timelines = (mc.n_pre_layers ? 1 : 0) + S +
                            (mc.n_post_layers ? (int)endpoint_kind.size() : 0);
    if (sc.request_rows > 0) {
      rows = sc.request_rows;
    } else {
      // schedule bound of pipeline.py:195-230 plus the prompt timelines
      std::vector<long> births = birth_sizes();
      births.push_back(X == 0 ? 1 : births.back() + births[depth - X]);
      std::vector<int> post_steps;
      for (auto& e : endpoint_kind) post_steps.push_back(e.first / K + 1);
      const int hp = mc.n_pre_layers ? 1 : 0, hq = mc.n_post_layers ? 1 : 0;
      long total = 2L * (S + hp + hq * (long)post_steps.size());
      for (int age = 1; age <= depth; ++age) {
        int reached = 0;
        for (int st : post_steps) reached += st <= age;
        total += births[depth + 1 - age] * (K * age + hp + hq * reached);
      }
      rows = (int)total + n_timelines;
    }
    if (sc.kv_slots > 0) {
      n_slots = sc.kv_slots;
    } else {
      n_slots = n_timelines * (max_ctx + 2 * max_rows) + 2 * rows;
    }
    // The device loop hands out KV slots without recycling them during a
    // request: each cycle takes one per lane per role call with attention,
    // and a token takes at most S / K cycles, so it needs up to
    // (S / K) * max_ctx * max_rows * (K + pre + post) slots beyond the prompt.
    // It is used only while that pool stays modest (24 GB of K/V).
    loop_enabled = false;
    if (device_loop_possible()) {
      const long roles = K + (mc.n_pre_layers ? 1 : 0) + (mc.n_post_layers ? 1 : 0);
      const long need = (long)(S / K) * max_ctx * max_rows * roles + (long)n_timelines * max_ctx;
      const double kv_bytes = 2.0 * (mc.n_pre_layers + mc.n_core_layers + mc.n_post_layers) *
                              (double)std::max<long>(need, n_slots) * (mc.n_kv_heads * mc.head_dim) * 2.0;
      if (sc.kv_slots <= 0 && max_req == 1 && kv_bytes <= 24e9) {
        n_slots = (int)std::max<long>(need, n_slots);
        loop_enabled = true;
      }
    }
    // per-request capacities (request_rows / kv_slots size one request),
    // disjoint ranges per request
    reqs.assign(max_req, Request());
    for (int i = 0; i < max_req; ++i) {
      reqs[i].tl.configure(rows, n_slots, i * rows, i * n_slots);
      reqs[i].state_base = i * max_rows;
    }
    rows *= max_req;
    n_slots *= max_req;

    // weights
    embed = W("pre_executor.embed_tokens.weight", {V, H});
    lm_head = mc.tie_embeddings ? embed : W("post_executor.lm_head.weight", {V, H});
    load_stack(pre, "pre_executor.blocks.", mc.n_pre_layers);
    load_stack(core, "recurrent_executor.blocks.", mc.n_core_layers);
    load_stack(post, "post_executor.blocks.", mc.n_post_layers);
    pre.kv_base = 0;
    core.kv_base = mc.n_pre_layers;
    post.kv_base = mc.n_pre_layers + mc.n_core_layers;
    if (mc.family == LS_FAMILY_OURO) {
      step_norm = W("recurrent_executor.step_norm.weight", {H});
    } else {
      g_adapter = cluster_gemm(W("recurrent_executor.adapter.weight", {H, 2 * H}), H, 2 * H);
      if (mc.adapter_bias) adapter_b = W("recurrent_executor.adapter.bias", {H});
      final_norm = W("post_executor.final_norm.weight", {H});
    }
    g_lm = make_gemm(lm_head, V, H, 1);
    REQUIRE(mc.n_core_layers > 0, LS_EINVAL, "core needs at least one layer");

    // device memory
    const long kv_elems = (long)n_attn_layers * n_slots * KVD;
    kpool = dalloc<bf16>(kv_elems);
    vpool = dalloc<bf16>(kv_elems);
    map = dalloc<int>((long)rows * max_ctx);
    bank_h = dalloc<float>((long)bank_rows * H);
    bank_inj = dalloc<float>((long)bank_rows * H);
    meta_dev = dalloc<int>(3L * kMetaFields * cap);
    if (loop_enabled) {
      loop_sched = dalloc<LoopSched>(1);
      CK(cudaMallocHost(&loop_host, sizeof(LoopSched)));
      loop_meta = dalloc<int>((long)(K + 2) * kMetaFields * cap);
      loop_active = dalloc<int>(3);
      loop_out = dalloc<long long>(max_ctx);
    }
    CK(cudaMallocHost(&meta_host, sizeof(int) * (size_t)kStaging * kMetaFields * cap));
    h = dalloc<float>((long)cap * H);
    r = dalloc<float>((long)cap * H);
    q = dalloc<float>((long)cap * QD);
    part = dalloc<float>(part_elems);
    o_part = dalloc<float>((long)cap * NH * max_chunks * HD);
    ml_part = dalloc<float>((long)cap * NH * max_chunks * 2);
    logits = dalloc<float>((long)cap * V);
    const int xrows = round_up(2 * cap, 256);  // (hi, lo) row pair per lane
    auto mkx = [&](XBuf& xb, int Kd) {
      xb.K = Kd;
      xb.rows = xrows;
      xb.ptr = dalloc<bf16>((long)xrows * Kd);
    };
    mkx(x_h, H);
    mkx(x_attn, QD);
    mkx(x_act, I);
    if (mc.family == LS_FAMILY_RAVEN) mkx(x_cat, 2 * H);
    amax_dev = dalloc<long long>(cap);
    amax_val = dalloc<float>((long)cap * cdiv(V, kGemmBM));
    amax_idx = dalloc<int>((long)cap * cdiv(V, kGemmBM));
    amax_ticket = dalloc<int>(1);
    CK(cudaMallocHost(&amax_host, sizeof(long long) * cap));
    CK(cudaMallocHost(&logits_host, sizeof(float) * (size_t)V));
    err_dev = dalloc<int>(1);
    attn_tickets = dalloc<int>((long)cap * NKV);
    gemm_part = dalloc<float>(gemm_part_elems);
    // one parameter slot per request (slot i: request i; single-request calls use slot 0)
    sparams_dev = dalloc<SampleParams>(max_req);
    for (int i = 0; i < max_req; ++i)
      CK(cudaMemcpy(sparams_dev + i, &sparams, sizeof(SampleParams), cudaMemcpyHostToDevice));
    q1_bank = dalloc<float>((long)max_state * V);
    r_bank = dalloc<float>((long)max_state * V);
    dec_dev = dalloc<long long>((long)cap * 5);
    CK(cudaMallocHost(&dec_host, sizeof(long long) * 5 * (size_t)cap));
    CK(cudaMallocHost(&err_host, sizeof(int)));
    REQUIRE(V <= kSampleChunk * kSampleMaxChunks, LS_EINVAL, "vocabulary above the sampler's limit");
    CK(cudaFuncSetAttribute(sample_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                            (int)sample_smem_bytes(V)));
    CK(cudaFuncSetAttribute(sample_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                            (int)sample_smem_bytes(V)));
    CK(cudaFuncSetAttribute(prefill_attn_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                            (int)pattn_smem_bytes<128>()));
    CK(cudaFuncSetAttribute(prefill_attn_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                            (int)pattn_smem_bytes<64>()));
    gemm_tickets = dalloc<int>(gemm_ticket_count);
    std::vector<float> inv(HD / 2);
    for (int i = 0; i < HD / 2; ++i)
      inv[i] = (float)(1.0 / std::pow((double)mc.rope_theta, (2.0 * i) / HD));
    inv_freq = dalloc<float>(HD / 2);
    CK(cudaMemcpy(inv_freq, inv.data(), sizeof(float) * inv.size(), cudaMemcpyHostToDevice));

    set_smem_attrs();
    finalized = true;
  }

  std::vector<long> birth_sizes() const {
    std::vector<long> b;
    if (X == 0) {
      b.assign(depth, 1);
    } else {
      b.assign(X, 1);
      for (int t = X; t < depth; ++t) b.push_back(b[t - 1] + b[t - X]);
    }
    return b;
  }

  void set_smem_attrs() {
#define LS_SMEM1(BN, ST, EPI)                                                                   \
  CK(cudaFuncSetAttribute(gemm_tc_kernel<BN, ST, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                          GemmSmem<BN, ST>::kTotal))
#define LS_SMEM(BN, ST)          \
  LS_SMEM1(BN, ST, kEpiStore);   \
  LS_SMEM1(BN, ST, kEpiQkvRope); \
  LS_SMEM1(BN, ST, kEpiSwiGLU);  \
  LS_SMEM1(BN, ST, kEpiSplitStore);  \
  LS_SMEM1(BN, ST, kEpiStoreArgmax); \
  LS_SMEM1(BN, ST, kEpiClusterStore); \
  CK(cudaFuncSetAttribute(gemm_tc_kernel<BN, ST, kEpiClusterStore>,  \
                          cudaFuncAttributeNonPortableClusterSizeAllowed, 1))
    LS_SMEM(16, 4);
    LS_SMEM(32, 4);
    LS_SMEM(64, 4);
    LS_SMEM(128, 3);
    LS_SMEM(256, 2);
#undef LS_SMEM
#undef LS_SMEM1
    const int row_smem = std::max(QD + 2 * KVD, 2 * H) * (int)sizeof(float);
    CK(cudaFuncSetAttribute(qkv_epi_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, row_smem));
  }
};

// ============================================================ role kernel chains
namespace {

Meta meta_of(ls_engine& e, int role) {
  if (e.meta_override) return Meta{e.meta_override, e.cap};
  return Meta{e.meta_dev + (long)role * kMetaFields * e.cap, e.cap};
}

int pick_bn(int n) {
  if (n <= 16) return 16;
  if (n <= 32) return 32;
  if (n <= 64) return 64;
  if (n <= 128) return 128;
  return 256;
}

// n lanes = 2n activation rows (hi/lo pairs) starting at lane `lane0`.
// Launch one weight-streaming GEMM over n lanes (2n activation rows, hi/lo
// pairs) starting at lane `lane0`, as (m_tiles, splits, n_tiles) CTAs in
// clusters of (1, splits, 1).
void gemm(ls_engine& e, const Gemm& g, XBuf& x, const GemmEpi& epi, int kind, int n,
          int lane0 = 0) {
  REQUIRE(n >= 1 && 2 * (lane0 + n) <= x.rows, LS_EINVAL, "GEMM lane count out of range");
  REQUIRE(g.splits >= 1 && g.splits <= kMaxSplits, LS_EINVAL, "bad split count");
  REQUIRE(kind != kEpiStoreArgmax || (g.splits == 1 && g.Mw <= e.V), LS_EINVAL,
          "the fused argmax needs an unsplit GEMM of at most vocab rows");
  // prefill: the wide QKV and gate_up projections run unsplit, on N tiles of
  // at most 64 lanes so that each weight tile is shared by two CTAs
  const bool unsplit = e.prefill_mode && (kind == kEpiQkvRope || kind == kEpiSwiGLU);
  const int splits = unsplit ? 1 : g.splits;
  REQUIRE(kind != kEpiSwiGLU || g.has_map64, LS_EINVAL, "SwiGLU needs the 64-row weight map");
  const int bn = unsplit ? std::min(pick_bn(2 * n), 128) : pick_bn(2 * n);
  const CUtensorMap& xm = x.map(bn);
  const int x_row0 = 2 * lane0;
  const int m_tiles = kind == kEpiSwiGLU ? g.Mw / kGemmBM : cdiv(g.Mw, kGemmBM);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(m_tiles, splits, cdiv(2 * n, bn));
  cfg.blockDim = dim3(kGemmThreads);
  cfg.stream = e.stream;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (kind == kEpiClusterStore) {   // the K splits of a tile form one cluster
    REQUIRE(splits >= 1 && splits <= kMaxClusterSplits, LS_EINVAL, "cluster store needs <= 16 splits");
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = 1;
    attr[na].val.clusterDim.y = (unsigned)splits;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  if (e.sc.use_pdl && !e.serialize_next) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  e.serialize_next = false;
  GemmEpi ep = epi;
  ep.active = e.gemm_active;
  ep.part_ws = e.gemm_part;
  ep.tile_tickets = e.gemm_tickets;
  REQUIRE(splits == 1 || kind == kEpiClusterStore ||
              (long)cfg.gridDim.x * cfg.gridDim.z <= e.gemm_ticket_count, LS_EINVAL, "GEMM tile tickets too small");
  REQUIRE((long)cfg.gridDim.x * cfg.gridDim.z * splits * (bn / 2) * kGemmBM <= e.gemm_part_elems ||
              splits == 1 || kind == kEpiClusterStore, LS_EINVAL, "GEMM partial scratch too small");
  const CUtensorMap& wm = kind == kEpiSwiGLU ? g.map64 : g.map;
#define LS_GEMM_K(BN, ST, EPI)                                                                     \
  do {                                                                                              \
    cfg.dynamicSmemBytes = GemmSmem<BN, ST>::kTotal;                                                \
    CK(cudaLaunchKernelEx(&cfg, gemm_tc_kernel<BN, ST, EPI>, wm, xm, ep, g.Mw, g.K, n, x_row0, \
                          splits, e.err_dev));                                                     \
  } while (0)
#define LS_GEMM(BN, ST)                                           \
  do {                                                            \
    if (kind == kEpiQkvRope) LS_GEMM_K(BN, ST, kEpiQkvRope);      \
    else if (kind == kEpiSwiGLU) LS_GEMM_K(BN, ST, kEpiSwiGLU);   \
    else if (kind == kEpiSplitStore) LS_GEMM_K(BN, ST, kEpiSplitStore); \
    else if (kind == kEpiClusterStore) LS_GEMM_K(BN, ST, kEpiClusterStore); \
    else if (kind == kEpiStoreArgmax) LS_GEMM_K(BN, ST, kEpiStoreArgmax); \
    else LS_GEMM_K(BN, ST, kEpiStore);                            \
  } while (0)
  switch (bn) {
    case 16: LS_GEMM(16, 4); break;
    case 32: LS_GEMM(32, 4); break;
    case 64: LS_GEMM(64, 4); break;
    case 128: LS_GEMM(128, 3); break;
    default: LS_GEMM(256, 2); break;
  }
#undef LS_GEMM
#undef LS_GEMM_K
  e.kernels_in_call++;
}

GemmEpi store_to(float* out) {
  GemmEpi ep{};
  ep.out = out;
  return ep;
}

void gemm_store(ls_engine& e, const Gemm& g, XBuf& x, float* out, int n, int lane0 = 0) {
  gemm(e, g, x, store_to(out), kEpiStore, n, lane0);
}

// y as partial planes [plane][cap][Mw] in e.part (or `planes`) for a
// consumer that adds them in plane order. For a cluster GEMM (O, down,
// adapter) the splits of each tile add their partials inside the GEMM through
// distributed shared memory and leave one plane (plane_count); otherwise each
// split writes its own plane (no split-K ticket or re-read either way).
void gemm_split_store(ls_engine& e, const Gemm& g, XBuf& x, int n, float* planes = nullptr) {
  GemmEpi ep = store_to(planes ? planes : e.part);
  ep.split_stride = (long)e.cap * g.Mw;
  gemm(e, g, x, ep, g.cluster && !planes ? kEpiClusterStore : kEpiSplitStore, n);
}

// Planes gemm_split_store leaves in e.part for its consumer.
int plane_count(const Gemm& g) { return g.cluster ? 1 : g.splits; }

template <typename... KArgs, typename... Args>
void klaunch(ls_engine& e, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
             Args&&... args) {
  launch(kernel, grid, block, smem, e.stream, e.sc.use_pdl != 0 && !e.serialize_next,
         std::forward<Args>(args)...);
  e.serialize_next = false;
  e.kernels_in_call++;
}

// klaunch for a kernel of thread-block clusters of `cluster` CTAs along x.
template <typename... KArgs, typename... Args>
void klaunch_cluster(ls_engine& e, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                     int cluster, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = e.stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)cluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = e.sc.use_pdl != 0 && !e.serialize_next ? 2 : 1;
  CK(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...));
  e.serialize_next = false;
  e.kernels_in_call++;
}

void map_update(ls_engine& e, Meta meta, int n) {
  klaunch(e, map_update_kernel, dim3(n), dim3(128), 0, meta, n, e.map, e.max_ctx, e.rows, e.err_dev);
  // attention reads slot ids before its wait (a forking lane after it):
  // unless the update only appends each lane's new position and every
  // attention layer takes it from the metadata (decode form, no QK-norm
  // layer), later kernels start after it has completed
  e.serialize_next = !e.qkv_planes || e.mc.qk_norm != 0;
}

// Threads of a per-lane row kernel: one float4 column each, at most 1024.
int row_threads(int H) { return std::min(1024, H / 4); }

template <int FORM>
void launch_attention(ls_engine& e, dim3 grid, dim3 blk, int G, const AttnArgs& a) {
  if (e.HD == 128 && G == 1) klaunch(e, attn_kernel<128, 1, FORM>, grid, blk, 0, a);
  else if (e.HD == 128 && G == 2) klaunch(e, attn_kernel<128, 2, FORM>, grid, blk, 0, a);
  else if (e.HD == 64 && G == 1) klaunch(e, attn_kernel<64, 1, FORM>, grid, blk, 0, a);
  else if (e.HD == 64 && G == 2) klaunch(e, attn_kernel<64, 2, FORM>, grid, blk, 0, a);
  else klaunch(e, attn_kernel<64, 4, FORM>, grid, blk, 0, a);
}

// Attention form for a grid of `ctas` CTAs on `sms` SMs (measured on
// Ouro-1.4B core calls: the early forms win up to two CTAs per SM, the
// late-V form above; the wide-register form only while every CTA can be
// resident beside the projection that precedes it).
int attention_form(long ctas, int sms) {
  return ctas <= sms ? kAttnWide : ctas <= 2L * sms ? kAttnMid : kAttnVLate;
}

// planes: the QKV projection's split planes (decode form), or null when the
// projection's epilogue already wrote q and the new K/V.
void attention(ls_engine& e, Meta meta, int n, bf16* kp, bf16* vp, const Gemm* planes = nullptr) {
  AttnArgs a{meta, e.NH, e.NKV, e.q, e.map, e.max_ctx, e.rows, kp, vp, e.n_slots,
             e.max_chunks, e.o_part, e.ml_part, e.attn_tickets, e.x_attn.ptr, nullptr,
             nullptr, nullptr, 1.0f / std::sqrt((float)e.HD), e.err_dev};
  if (planes) {
    a.qkv = e.part;
    a.qkv_splits = plane_count(*planes);
    a.qkv_stride = (long)e.cap * planes->Mw;
    a.inv_freq = e.inv_freq;
    a.kpool_w = kp;
    a.vpool_w = vp;
  }
  if (!planes && e.prefill_mode && (e.HD == 128 || e.HD == 64)) {
    // a prompt chunk of one timeline: tensor-core tiles over the shared K/V
    const dim3 pg(cdiv(n, kPAttnRows), e.NH), pb(kPAttnThreads);
    if (e.HD == 128) klaunch(e, prefill_attn_kernel<128>, pg, pb, pattn_smem_bytes<128>(), a, n);
    else klaunch(e, prefill_attn_kernel<64>, pg, pb, pattn_smem_bytes<64>(), a, n);
    return;
  }
  const dim3 grid(n, e.NKV, e.attn_chunks), blk(kAttnThreads);
  const int G = e.NH / e.NKV;
  const long form_lanes = e.attn_form_lanes > 0 ? std::min(n, e.attn_form_lanes) : n;
  const int form = attention_form(form_lanes * e.NKV * e.attn_chunks, e.num_sms);
  if (form == kAttnWide) launch_attention<kAttnWide>(e, grid, blk, G, a);
  else if (form == kAttnMid) launch_attention<kAttnMid>(e, grid, blk, G, a);
  else launch_attention<kAttnVLate>(e, grid, blk, G, a);
}

ResidArgs resid_base(ls_engine& e, Meta meta, const Gemm& g) {
  ResidArgs a{};
  a.meta = meta;
  a.H = e.H;
  a.part = e.part;   // the GEMM's split planes (gemm_split_store)
  a.splits = plane_count(g);   // (the TP exchange keeps every split's plane)
  a.split_stride = (long)e.cap * g.Mw;
  a.bank_rows = e.bank_rows;
  a.eps = e.mc.rms_eps;
  a.err = e.err_dev;
  return a;
}

void resid(ls_engine& e, ResidArgs a, int n) {
  a.B = n;
  const int thr = row_threads(e.H);
  const dim3 grid(n);
  if (a.tp.ranks > 1) {
    if (cdiv(e.H / 4, thr) > 1) klaunch(e, resid_epi_kernel<2, 4, 1024, true>, grid, dim3(thr), 0, a);
    else if (thr <= 512) klaunch(e, resid_epi_kernel<1, 10, 512, true>, grid, dim3(thr), 0, a);
    else klaunch(e, resid_epi_kernel<1, 8, 1024, true>, grid, dim3(thr), 0, a);
  } else if (cdiv(e.H / 4, thr) > 1) {
    klaunch(e, resid_epi_kernel<2, 4, 1024, false>, grid, dim3(thr), 0, a);
  } else if (thr <= 512) {
    klaunch(e, resid_epi_kernel<1, 10, 512, false>, grid, dim3(thr), 0, a);
  } else {
    klaunch(e, resid_epi_kernel<1, 8, 1024, false>, grid, dim3(thr), 0, a);
  }
}

// ------------------------------------------------------- tensor parallelism
constexpr size_t kTpEpochOff = 64;    // byte offset of the epoch counter in a region
constexpr size_t kTpTicketOff = 128;  // this rank's publish tickets, one per slot (not read by peers)

// Every rank's buffer at byte offset `off` of its region, in rank order.
TpView tp_view(const ls_engine& e, size_t off) {
  TpView t{};
  t.ranks = e.tp_ranks;
  t.wait_ns = e.tp_wait_ns;
  t.epoch = reinterpret_cast<const int*>(e.tp_region + kTpEpochOff);
  for (int r = 0; r < e.tp_ranks; ++r) {
    t.flags[r] = reinterpret_cast<const int*>(e.tp_base[r]);
    t.data[r] = reinterpret_cast<const float*>(e.tp_base[r] + off);
  }
  return t;
}

void tp_publish(ls_engine& e, int slot) {
  klaunch(e, tp_publish_kernel, dim3(1), dim3(32), 0, reinterpret_cast<int*>(e.tp_region + kTpEpochOff),
          reinterpret_cast<int*>(e.tp_region), slot);
}

// A row-sharded projection (O or down): this rank's split planes go to its
// exchange region and are published; the residual kernel that follows adds
// every rank's planes.
// The GEMM's last CTA publishes (no separate publish launch).
void tp_split_store(ls_engine& e, const Gemm& g, XBuf& x, int n, ResidArgs& ra, size_t off, int slot) {
  GemmEpi ep = store_to(reinterpret_cast<float*>(e.tp_region + off));
  ep.split_stride = (long)e.cap * g.Mw;
  ep.pub_epoch = reinterpret_cast<int*>(e.tp_region + kTpEpochOff);
  ep.pub_flag = reinterpret_cast<int*>(e.tp_region) + slot;
  ep.pub_ticket = reinterpret_cast<int*>(e.tp_region + kTpTicketOff) + slot;
  gemm(e, g, x, ep, kEpiSplitStore, n);
  ra.tp = tp_view(e, off);
  ra.splits = g.splits;
  ra.tp_slot = slot;
}

// Norm applied to the input of a layer's first GEMM (none for OLMo2 post-norm).
const bf16* input_norm(const ls_engine& e, const LayerW& w) {
  return e.mc.layout == LS_LAYOUT_OLMO_POST ? nullptr : w.n_in;
}

// One stack of decoder layers over n lanes. Input: h (fp32) and x_h = bf16 of
// the first layer's normalised input. Layer formulas:
//   ouro      r = h + rms(attn(rms(h)*n_in))*n_pa ; h = r + rms(mlp(rms(r)*n_pf))*n_pff
//   raven_pre r = h + attn(rms(h)*n_in)           ; h = r + mlp(rms(r)*n_pa)
//   olmo_post r = h + rms(attn(h))*n_pa           ; h = r + rms(mlp(r))*n_pff
// (ouro.py:37-82 over SGLang Gemma2DecoderLayer; raven.py:258-265 / Llama;
//  Olmo2DecoderLayer, contracts.py:191-196.)
void run_stack(ls_engine& e, Stack& st, int n, Meta meta, const StackEnd& end) {
  const int L = e.mc.layout;
  const int nl = (int)st.layers.size();
  for (int l = 0; l < nl; ++l) {
    LayerW& w = st.layers[l];
    const long kvoff = (long)(st.kv_base + l) * e.n_slots * e.KVD;
    bf16* kp = e.kpool + kvoff;
    bf16* vp = e.vpool + kvoff;

    if (w.qn) {
      // OLMo2 QK-norm needs whole-row sums: plain GEMM, then the QKV kernel.
      gemm_split_store(e, w.g_qkv, e.x_h, n);
      QkvArgs qa{meta, e.NH, e.NKV, e.HD, e.part, plane_count(w.g_qkv), (long)e.cap * w.g_qkv.Mw,
                 w.qn, w.kn, e.inv_freq, e.mc.rms_eps,
                 e.q, kp, vp, e.n_slots, e.err_dev};
      const size_t smem = (size_t)(e.QD + 2 * e.KVD) * sizeof(float);
      if (e.tp_ranks > 1) {
        // the norm spans every rank's heads: exchange the sums of squares
        qa.tp = tp_view(e, e.tp_off_qk);
        qa.tp_sums = reinterpret_cast<float*>(e.tp_region + e.tp_off_qk);
        qa.tp_phase = 1;
        klaunch(e, qkv_epi_kernel, dim3(n), dim3(256), smem, qa);
        tp_publish(e, kTpSlotQk);
        qa.tp_phase = 2;
      }
      klaunch(e, qkv_epi_kernel, dim3(n), dim3(256), smem, qa);
    } else if (e.qkv_planes) {
      // decode: split planes; attention sums them and does RoPE / the KV write
      gemm_split_store(e, w.g_qkv, e.x_h, n);
    } else {
      // RoPE and the K/V cache write run in the GEMM's reduction epilogue.
      GemmEpi ep{};
      ep.meta = meta.p;
      ep.inv_freq = e.inv_freq;
      ep.q = e.q;
      ep.kpool = kp;
      ep.vpool = vp;
      ep.hd = e.HD;
      ep.nh = e.NH;
      ep.nkv = e.NKV;
      ep.n_slots = e.n_slots;
      gemm(e, w.g_qkv, e.x_h, ep, kEpiQkvRope, n);
    }
    attention(e, meta, n, kp, vp, !w.qn && e.qkv_planes ? &w.g_qkv : nullptr);
    ResidArgs ra = resid_base(e, meta, w.g_o);
    if (e.tp_ranks > 1) tp_split_store(e, w.g_o, e.x_attn, n, ra, e.tp_off_o, kTpSlotO);
    else gemm_split_store(e, w.g_o, e.x_attn, n);
    ra.resid = e.h;
    ra.out_h = e.r;
    ra.x = e.x_h.ptr;
    if (L == LS_LAYOUT_OURO) {
      ra.a_norm_w = w.n_pa;
      ra.x_norm_w = w.n_pf;
    } else if (L == LS_LAYOUT_RAVEN_PRE) {
      ra.x_norm_w = w.n_pa;
    } else {
      ra.a_norm_w = w.n_pa;
    }
    resid(e, ra, n);

    // gate_up with SiLU(gate) * up fused into its epilogue -> x_act
    GemmEpi eg{};
    eg.x_act = e.x_act.ptr;
    eg.I = e.I;
    gemm(e, w.g_gu, e.x_h, eg, kEpiSwiGLU, n);
    ResidArgs rb = resid_base(e, meta, w.g_down);
    if (e.tp_ranks > 1) tp_split_store(e, w.g_down, e.x_act, n, rb, e.tp_off_d, kTpSlotDown);
    else gemm_split_store(e, w.g_down, e.x_act, n);
    rb.resid = e.r;
    rb.out_h = e.h;
    if (L != LS_LAYOUT_RAVEN_PRE) rb.a_norm_w = w.n_pff;
    const bool last = l + 1 == nl;
    if (!last) {
      rb.x = e.x_h.ptr;
      rb.x_norm_w = input_norm(e, st.layers[l + 1]);
    } else {
      rb.final_norm_w = end.final_norm;
      rb.bank = end.bank;
      if (end.want_x) {
        rb.x = e.x_h.ptr;
        rb.x_norm_w = end.x_norm;
      }
    }
    resid(e, rb, n);
  }
}

struct PostOpts {
  bool layers = true;     // run coda layers (post timelines)
  bool head = true;       // run lm_head + argmax
  int head_lane0 = 0;     // first lane of the head
  int head_lanes = -1;    // number of lanes through the head (-1: all)
};

void prep(ls_engine& e, Meta meta, int n, bool embed_mode, float* bank_out, bool want_x,
          const bf16* x_norm) {
  PrepArgs pa{};
  pa.meta = meta;
  pa.B = n;
  pa.H = e.H;
  pa.embed = embed_mode ? e.embed : nullptr;
  pa.embed_scale = e.mc.embed_scale;
  pa.bank_in = e.bank_h;
  pa.bank_rows = e.bank_rows;
  pa.h = e.h;
  pa.bank_out = bank_out;
  pa.x = want_x ? e.x_h.ptr : nullptr;
  pa.x_norm_w = x_norm;
  pa.eps = e.mc.rms_eps;
  pa.vocab = e.V;
  pa.err = e.err_dev;
  pa.meta_after_wait = e.meta_after_wait;
  e.meta_after_wait = 0;
  const int thr = row_threads(e.H);
  const dim3 grid(n);
  if (cdiv(e.H / 4, thr) == 1) klaunch(e, prep_kernel<1>, grid, dim3(thr), 0, pa);
  else klaunch(e, prep_kernel<2>, grid, dim3(thr), 0, pa);
}

// Readout decisions of the head lanes: fused sampler or greedy argmax.
void head_decisions(ls_engine& e, Meta meta, int lane0, int lanes) {
  if (e.sampling) {
    REQUIRE(lanes <= e.max_state, LS_ECAPACITY, "too many sampled readout rows");
    SampleArgs sa{meta, lane0, e.logits, e.V, e.sparams_dev, e.max_req, e.q1_bank, e.r_bank,
                  e.max_state, e.dec_dev, e.err_dev};
    // one cluster of CTAs per row; rows in 16-byte steps when the vocabulary
    // allows (logits and bank rows are then 16-byte aligned)
    const int C = sample_ctas(e.V);
    const dim3 g(lanes * C), b(kSampleThreads);
    const size_t smem = sample_smem_bytes(e.V);
    if (e.V % 4 == 0) klaunch_cluster(e, sample_kernel<4>, g, b, smem, C, sa);
    else klaunch_cluster(e, sample_kernel<1>, g, b, smem, C, sa);
  } else {
    klaunch(e, argmax_kernel, dim3(lanes), dim3(1024), 0, (const float*)e.logits, e.V, (long)e.V,
            e.amax_dev);
  }
}

// The kernel chain of one role call over n lanes whose metadata is in the
// role's device metadata buffer.
void enqueue_role(ls_engine& e, int role, int n, const PostOpts& po = PostOpts()) {
  Meta meta = meta_of(e, role);
  e.kernels_in_call = 0;
  const bool ouro = e.mc.family == LS_FAMILY_OURO;
  if (role == kPre) {
    if (ouro) {
      // Ouro pre = embedding only (ouro.py:101-136); write it to the bank.
      prep(e, meta, n, true, e.bank_h, false, nullptr);
    } else {
      // Raven pre: embed*scale, prelude, then the position-keyed hidden init
      // with the prelude output kept as the injection (components.py:117-149).
      if (!e.pre.layers.empty()) map_update(e, meta, n);
      prep(e, meta, n, true, nullptr, !e.pre.layers.empty(),
           e.pre.layers.empty() ? nullptr : input_norm(e, e.pre.layers[0]));
      if (!e.pre.layers.empty()) run_stack(e, e.pre, n, meta, StackEnd());
      klaunch(e, raven_init_kernel, dim3(n), dim3(256), 0, meta, e.H, (const float*)e.h, e.bank_h,
              e.bank_inj, e.bank_rows, (unsigned long long)e.mc.init_seed, e.mc.init_std,
              e.mc.embed_scale, e.err_dev);
    }
  } else if (role == kCore) {
    map_update(e, meta, n);
    StackEnd end;
    end.bank = e.bank_h;
    if (ouro) {
      // one core iteration = all layers then step_norm (ouro.py:93-98)
      prep(e, meta, n, false, nullptr, true, input_norm(e, e.core.layers[0]));
      end.final_norm = e.step_norm;
    } else {
      // adapter(cat(hidden, injected)) then the core blocks (raven.py:271-281)
      klaunch(e, cat_state_kernel, dim3(n), dim3(256), 0, meta, e.H, (const float*)e.bank_h,
              (const float*)e.bank_inj, e.bank_rows, e.x_cat.ptr, e.err_dev);
      gemm_split_store(e, e.g_adapter, e.x_cat, n);
      ResidArgs ra = resid_base(e, meta, e.g_adapter);
      ra.bias = e.adapter_b;
      ra.out_h = e.h;
      ra.x = e.x_h.ptr;
      ra.x_norm_w = input_norm(e, e.core.layers[0]);
      resid(e, ra, n);
    }
    run_stack(e, e.core, n, meta, end);
  } else {
    // post: coda layers (own timelines), final norm, lm_head (components.py:175-194)
    const bool has_layers = !e.post.layers.empty();
    if (has_layers && po.layers) {
      map_update(e, meta, n);
      prep(e, meta, n, false, nullptr, true, input_norm(e, e.post.layers[0]));
      StackEnd end;
      end.want_x = true;
      end.x_norm = e.final_norm;
      run_stack(e, e.post, n, meta, end);
    } else if (!has_layers) {
      prep(e, meta, n, false, nullptr, true, e.final_norm);
    }
    if (po.head) {
      const int lanes = po.head_lanes < 0 ? n : po.head_lanes;
      if (e.sampling) {
        gemm_store(e, e.g_lm, e.x_h, e.logits, lanes, po.head_lane0);
        head_decisions(e, meta, po.head_lane0, lanes);
      } else {
        // greedy: the lm_head GEMM also reduces each lane's argmax
        GemmEpi ep = store_to(e.logits);
        ep.amax_val = e.amax_val;
        ep.amax_idx = e.amax_idx;
        ep.amax_ticket = e.amax_ticket;
        ep.amax_out = e.amax_dev;
        gemm(e, e.g_lm, e.x_h, ep, kEpiStoreArgmax, lanes, po.head_lane0);
      }
    }
  }
}

int* stage_meta(ls_engine& e) {
  if (e.staging_next >= ls_engine::kStaging) {
    CK(cudaStreamSynchronize(e.stream));
    e.staging_next = 0;
  }
  int* p = e.meta_host + (long)e.staging_next++ * kMetaFields * e.cap;
  std::fill(p, p + kMetaFields * e.cap, -1);
  return p;
}

void upload_meta(ls_engine& e, int role, const int* host, int n) {
  const size_t bytes = sizeof(int) * kMetaFields * (size_t)n;
  CK(cudaMemcpyAsync(e.meta_dev + (long)role * kMetaFields * e.cap, host, bytes,
                     cudaMemcpyHostToDevice, e.stream));
  e.h2d_bytes += (int64_t)bytes;
}

void run_role(ls_engine& e, int role, int n, const int* host_meta, bool graphable,
              const PostOpts& po = PostOpts()) {
  REQUIRE(n >= 1 && n <= e.cap, LS_ECAPACITY, "role call wider than the lane capacity");
  upload_meta(e, role, host_meta, n);
  int longest = 1;
  bool single = true;   // no lane shares its timeline with an earlier lane of the call
  bool forks = false;
  if (role == kPre && e.mc.n_pre_layers > 0) e.pre_calls++;
  if (role == kCore) e.core_calls++;
  if (role == kPost && po.head) e.post_calls++;
  for (int b = 0; b < n; ++b) {
    if (role == kCore) e.core_kv_positions += host_meta[b * kMetaFields + kMetaPos] + 1;
    longest = std::max(longest, host_meta[b * kMetaFields + kMetaPos] + 1);
    single = single && host_meta[b * kMetaFields + kMetaAhead] <= 0;
    forks = forks || host_meta[b * kMetaFields + kMetaForkRow] >= 0;
  }
  const int chunks = cdiv(longest, kAttnChunk);
  e.qkv_planes = single;
  if (!(graphable && e.sc.use_graphs)) {
    e.attn_chunks = std::min(chunks, e.max_chunks);
    enqueue_role(e, role, n, po);
    e.kernel_launches += e.kernels_in_call;
    return;
  }
  e.attn_chunks = std::min(chunks + (chunks & 1), e.max_chunks);
  const auto key = std::make_pair(role * 4 + (e.sampling ? 2 : 0) + (forks ? 1 : 0), n);
  auto it = e.graphs.find(key);
  if (it != e.graphs.end() && (e.graph_chunks[key] != e.attn_chunks || e.graph_planes[key] != e.qkv_planes)) {
    CK(cudaStreamSynchronize(e.stream));
    CK(cudaGraphExecDestroy(it->second));
    e.graphs.erase(it);
    it = e.graphs.end();
  }
  if (it == e.graphs.end()) {
    CK(cudaStreamBeginCapture(e.stream, cudaStreamCaptureModeThreadLocal));
    try {
      enqueue_role(e, role, n);
    } catch (...) {
      cudaGraph_t g = nullptr;
      cudaStreamEndCapture(e.stream, &g);
      if (g) cudaGraphDestroy(g);
      throw;
    }
    cudaGraph_t g = nullptr;
    CK(cudaStreamEndCapture(e.stream, &g));
    cudaGraphExec_t ge = nullptr;
    const cudaError_t ie = cudaGraphInstantiate(&ge, g, 0);
    cudaGraphDestroy(g);
    CK(ie);
    it = e.graphs.emplace(key, ge).first;
    e.graph_kernels[key] = e.kernels_in_call;
    e.graph_chunks[key] = e.attn_chunks;
    e.graph_planes[key] = e.qkv_planes;
  }
  CK(cudaGraphLaunch(it->second, e.stream));
  e.kernel_launches += e.graph_kernels[key];
}

void raise_device_error(ls_engine& e, int err);

void check_device(ls_engine& e) {
  int err = 0;
  CK(cudaMemcpy(&err, e.err_dev, sizeof(int), cudaMemcpyDeviceToHost));
  e.d2h_bytes += sizeof(int);
  raise_device_error(e, err);
}

// Per-step form: queue the error word's copy behind the step's kernels (no
// extra synchronisation), then, after the step's stream synchronisation,
// check_fetched_error() reads it.
void fetch_device_error(ls_engine& e) {
  CK(cudaMemcpyAsync(e.err_host, e.err_dev, sizeof(int), cudaMemcpyDeviceToHost, e.stream));
  e.d2h_bytes += sizeof(int);
}

void check_fetched_error(ls_engine& e) { raise_device_error(e, *e.err_host); }

void raise_device_error(ls_engine& e, int err) {
  if (err != kDevOk) {
    CK(cudaMemset(e.err_dev, 0, sizeof(int)));
    static const char* names[] = {"ok", "TMA stage wait timed out", "free-stage wait timed out",
                                  "accumulator wait timed out", "metadata index out of range",
                                  "unused (5)", "unused (6)",
                                  "tensor-parallel peer wait timed out"};
    throw EngineError(LS_EDEVICE, std::string("device reported: ") +
                                      (err > 0 && err < 8 ? names[err] : "unknown error"));
  }
}

}  // namespace

// ============================================================ request execution
namespace {

void put(ls_engine& e, int* m, int field, int b, int v) {
  (void)e;
  m[b * kMetaFields + field] = v;
}

// Fill one lane of a role call. With a cursor, allocate the KV slot that this
// token's K/V gets on that timeline (from the lane's request) and describe a
// pending fork copy. `ahead` counts lanes of the same timeline filled earlier
// in this call (prefill feeds a whole prompt chunk of one timeline at once).
// Returns the slot (or -1).
int fill_lane(ls_engine& e, Timelines& tl, int* m, int b, int token, int pos, Cursor* c, int state_in,
              int state_out, int ahead = 0) {
  put(e, m, kMetaToken, b, token);
  put(e, m, kMetaPos, b, pos);
  put(e, m, kMetaStateIn, b, state_in);
  put(e, m, kMetaStateOut, b, state_out);
  if (!c) return -1;
  REQUIRE(c->seq_len + ahead == pos, LS_EPIPELINE,
          "timeline length " + std::to_string(c->seq_len) + " does not match position " +
              std::to_string(pos));
  REQUIRE(pos < e.max_ctx, LS_ECAPACITY, "context longer than max_context");
  const int slot = tl.alloc_slot();
  put(e, m, kMetaRow, b, c->row);
  put(e, m, kMetaSlot, b, slot);
  put(e, m, kMetaForkRow, b, c->pending_parent_row);
  put(e, m, kMetaForkLen, b, c->pending_parent_row >= 0 ? c->seq_len : 0);
  put(e, m, kMetaAhead, b, ahead);
  return slot;
}

// After submission: the cursor owns its new slot and its fork is done
// (request.py:216-222).
void advance(Cursor* c, int slot, bool owned) {
  if (owned) c->owned.push_back(slot);
  c->pending_parent_row = -1;
  c->seq_len += 1;
}

// The random stream of a readout row: the request's seed and cycle counter,
// and the row's index among the request's readouts of that cycle.
void set_draw(ls_engine& e, int* m, int b, const Request& R, int draw, int draw_row) {
  put(e, m, kMetaReq, b, (int)(&R - e.reqs.data()));
  put(e, m, kMetaCycle, b, draw);
  put(e, m, kMetaDrawRow, b, draw_row);
  put(e, m, kMetaSeedLo, b, (int)(uint32_t)(R.seed & 0xFFFFFFFFull));
  put(e, m, kMetaSeedHi, b, (int)(uint32_t)(R.seed >> 32));
}

// A readout that only draws the next token (no proposal to verify).
void set_final_readout(ls_engine& e, int* m, int b, const Request& R, int draw, int draw_row) {
  put(e, m, kMetaKind, b, 2);
  put(e, m, kMetaFirst, b, -1);
  put(e, m, kMetaSecond, b, -1);
  set_draw(e, m, b, R, draw, draw_row);
}

long long prefill(ls_engine& e, Request& R, const int64_t* prompt, int P, float* logits_out) {
  REQUIRE(e.finalized, LS_EINVAL, "engine not finalized");
  REQUIRE(P >= 1 && P <= e.sc.max_prompt, LS_EINVAL, "prompt length out of range");
  for (int i = 0; i < P; ++i)
    REQUIRE(prompt[i] >= 0 && prompt[i] < e.V, LS_EINVAL, "prompt token out of vocabulary");
  CK(cudaSetDevice(e.device));
  CK(cudaStreamSynchronize(e.stream));
  Timelines& tl = R.tl;
  tl.reset();
  e.staging_next = 0;
  R.prefill_len = P - 1;
  R.draw_cycle = 0;   // the first token uses draw 0, decode cycles 1, 2, ...
  CK(cudaMemsetAsync(e.err_dev, 0, sizeof(int), e.stream));
  CK(cudaEventRecord(e.ev0, e.stream));
  struct PrefillMode {   // unsplit wide projections while prefill enqueues (see prefill_mode)
    ls_engine& e;
    explicit PrefillMode(ls_engine& x) : e(x) { e.prefill_mode = true; }
    ~PrefillMode() { e.prefill_mode = false; }
  } prefill_scope(e);

  const bool pre_attn = e.mc.n_pre_layers > 0, post_attn = e.mc.n_post_layers > 0;
  Cursor* pre_c = pre_attn ? tl.create_root_cursor(kPre, 0) : nullptr;
  std::vector<Cursor*> core_c(e.S);
  for (int s = 0; s < e.S; ++s) core_c[s] = tl.create_root_cursor(kCore, s);
  std::map<int, Cursor*> post_c;
  if (post_attn)
    for (auto& ep : e.endpoint_kind) post_c[ep.first] = tl.create_root_cursor(kPost, ep.first);

  // prompt lanes use the scratch bank rows after every request's state slots
  const int scratch = e.max_state;
  const int chunk = e.prefill_chunk;
  for (int c0 = 0; c0 < P; c0 += chunk) {
    const int n = std::min(chunk, P - c0);
    const bool last_chunk = c0 + n == P;
    std::vector<int> slots(n);
    int* m = stage_meta(e);
    for (int j = 0; j < n; ++j)
      slots[j] = fill_lane(e, tl, m, j, (int)prompt[c0 + j], c0 + j, pre_c, -1, scratch + j, j);
    run_role(e, kPre, n, m, false);
    if (pre_c)
      for (int j = 0; j < n; ++j) advance(pre_c, slots[j], false);
    for (int s = 0; s < e.S; ++s) {
      m = stage_meta(e);
      for (int j = 0; j < n; ++j)
        slots[j] = fill_lane(e, tl, m, j, (int)prompt[c0 + j], c0 + j, core_c[s], scratch + j,
                             scratch + j, j);
      run_role(e, kCore, n, m, false);
      for (int j = 0; j < n; ++j) advance(core_c[s], slots[j], false);
      if (post_attn && e.endpoint_kind.count(s)) {
        m = stage_meta(e);
        for (int j = 0; j < n; ++j)
          slots[j] = fill_lane(e, tl, m, j, 0, c0 + j, post_c[s], scratch + j, -1, j);
        PostOpts po;
        po.head = last_chunk && s == e.S - 1;
        po.head_lane0 = n - 1;
        po.head_lanes = 1;
        if (po.head) set_final_readout(e, m, n - 1, R, 0, 0);
        run_role(e, kPost, n, m, false, po);
        for (int j = 0; j < n; ++j) advance(post_c[s], slots[j], false);
      }
    }
    if (!post_attn && last_chunk) {
      m = stage_meta(e);
      fill_lane(e, tl, m, 0, 0, P - 1, nullptr, scratch + n - 1, -1);
      set_final_readout(e, m, 0, R, 0, 0);
      run_role(e, kPost, 1, m, false);
    }
  }
  CK(cudaEventRecord(e.ev1, e.stream));
  if (e.sampling)
    CK(cudaMemcpyAsync(e.amax_host, e.dec_dev, sizeof(long long), cudaMemcpyDeviceToHost, e.stream));
  else
    CK(cudaMemcpyAsync(e.amax_host, e.amax_dev, sizeof(long long), cudaMemcpyDeviceToHost, e.stream));
  e.d2h_bytes += sizeof(long long);
  if (logits_out)
    CK(cudaMemcpyAsync(e.logits_host, e.logits, sizeof(float) * e.V, cudaMemcpyDeviceToHost, e.stream));
  CK(cudaStreamSynchronize(e.stream));
  e.staging_next = 0;
  check_device(e);
  if (logits_out) std::memcpy(logits_out, e.logits_host, sizeof(float) * e.V);
  return e.amax_host[0];
}

struct CycleLane {
  int stage, index, token, branch, parent, state;   // state: global state slot
  int origin = -1;   // scheduler bookkeeping only (trace output)
  int first = -1;    // the lane's q1 token (-1: none)
  int second = -1;   // the lane's q2 token (-1: none)
  int req = 0;       // the lane's request (index into the engine's batch)
};

// One readout decision: (token, proposed, accepted_code, q1_rejected,
// q2_rejected) for sampling (policy.py:197-218); greedy fills [0] only.
typedef std::array<long long, 5> Dec;

// One pipeline cycle (executor.py:293-367 without the decision policy) over
// the lanes of one or more requests: pre for stage-0 lanes, K core iterations
// for all lanes, post + decision for readout lanes, each role as one call
// over every request's lanes. dec[i] = the readout lane's decision, -1
// otherwise. Each request present advances its own random-stream cycle.
void cycle(ls_engine& e, const std::vector<CycleLane>& lanes, std::vector<Dec>& dec,
           float* logits_out) {
  const int B = (int)lanes.size();
  REQUIRE(B >= 1 && B <= e.max_state, LS_ECAPACITY, "speculative tree exceeded branch row limit");
  const bool pre_attn = e.mc.n_pre_layers > 0, post_attn = e.mc.n_post_layers > 0;
  std::vector<int> pos(B), pre_rows, ends(B), ep_rows;
  // random-stream index of this cycle's readouts: the request's pipeline
  // cycle number, counted whether or not the cycle has a readout
  std::vector<int> draw(e.reqs.size(), -1);
  for (int i = 0; i < B; ++i) {
    const CycleLane& l = lanes[i];
    REQUIRE(l.req >= 0 && l.req < (int)e.reqs.size(), LS_EINVAL, "lane request out of range");
    Request& R = e.reqs[l.req];
    REQUIRE(R.prefill_len >= 0, LS_EINVAL, "no prefilled request");
    REQUIRE(l.state >= R.state_base && l.state < R.state_base + e.max_rows, LS_EINVAL,
            "state slot out of range");
    REQUIRE(l.stage >= 0 && l.stage + e.K <= e.S && l.stage % e.K == 0, LS_EINVAL, "bad lane stage");
    REQUIRE(l.index >= 1, LS_EINVAL, "bad lane index");
    REQUIRE(l.token >= 0 && l.token < e.V, LS_EINVAL, "lane token out of vocabulary");
    pos[i] = R.prefill_len + l.index;
    ends[i] = l.stage + e.K - 1;
    if (l.stage == 0) pre_rows.push_back(i);
    if (e.endpoint_kind.count(ends[i])) ep_rows.push_back(i);
    if (draw[l.req] < 0) draw[l.req] = (int)(++R.draw_cycle);
  }
  std::vector<int> slots(B);
  if (!pre_rows.empty()) {
    int* m = stage_meta(e);
    std::vector<Cursor*> cs(pre_rows.size(), nullptr);
    for (size_t j = 0; j < pre_rows.size(); ++j) {
      const CycleLane& l = lanes[pre_rows[j]];
      Timelines& tl = e.reqs[l.req].tl;
      if (pre_attn) cs[j] = tl.get_or_create_cursor(kPre, 0, l.branch, l.parent);
      slots[j] = fill_lane(e, tl, m, (int)j, l.token, pos[pre_rows[j]], cs[j], -1, l.state);
    }
    run_role(e, kPre, (int)pre_rows.size(), m, true);
    for (size_t j = 0; j < pre_rows.size(); ++j)
      if (cs[j]) advance(cs[j], slots[j], true);
  }
  for (int off = 0; off < e.K; ++off) {
    int* m = stage_meta(e);
    std::vector<Cursor*> cs(B);
    for (int i = 0; i < B; ++i) {
      const CycleLane& l = lanes[i];
      Timelines& tl = e.reqs[l.req].tl;
      cs[i] = tl.get_or_create_cursor(kCore, l.stage + off, l.branch, l.parent);
      slots[i] = fill_lane(e, tl, m, i, l.token, pos[i], cs[i], l.state, l.state);
    }
    run_role(e, kCore, B, m, true);
    for (int i = 0; i < B; ++i) advance(cs[i], slots[i], true);
  }
  dec.assign(B, Dec{-1, 0, 0, 0, 0});
  if (ep_rows.empty()) return;
  const int M = (int)ep_rows.size();
  int* m = stage_meta(e);
  std::vector<Cursor*> cs(M, nullptr);
  std::vector<int> rows_of(e.reqs.size(), 0);   // readout rows per request so far
  for (int j = 0; j < M; ++j) {
    const CycleLane& l = lanes[ep_rows[j]];
    Request& R = e.reqs[l.req];
    if (post_attn) cs[j] = R.tl.get_or_create_cursor(kPost, ends[ep_rows[j]], l.branch, l.parent);
    slots[j] = fill_lane(e, R.tl, m, j, l.token, pos[ep_rows[j]], cs[j], l.state, -1);
    put(e, m, kMetaKind, j, e.endpoint_kind.at(ends[ep_rows[j]]));
    put(e, m, kMetaFirst, j, l.first);
    put(e, m, kMetaSecond, j, l.second);
    set_draw(e, m, j, R, draw[l.req], rows_of[l.req]++);
  }
  run_role(e, kPost, M, m, true);
  for (int j = 0; j < M; ++j)
    if (cs[j]) advance(cs[j], slots[j], true);
  if (e.sampling) {
    CK(cudaMemcpyAsync(e.dec_host, e.dec_dev, sizeof(long long) * 5 * M, cudaMemcpyDeviceToHost,
                       e.stream));
    e.d2h_bytes += sizeof(long long) * 5 * M;
  } else {
    CK(cudaMemcpyAsync(e.amax_host, e.amax_dev, sizeof(long long) * M, cudaMemcpyDeviceToHost,
                       e.stream));
    e.d2h_bytes += sizeof(long long) * M;
  }
  if (logits_out) {
    for (int j = 0; j < M; ++j)
      CK(cudaMemcpyAsync(logits_out + (long)ep_rows[j] * e.V, e.logits + (long)j * e.V,
                         sizeof(float) * e.V, cudaMemcpyDeviceToHost, e.stream));
  }
  fetch_device_error(e);
  CK(cudaStreamSynchronize(e.stream));
  e.host_syncs++;
  e.staging_next = 0;
  check_fetched_error(e);
  for (int j = 0; j < M; ++j) {
    if (e.sampling) {
      for (int f = 0; f < 5; ++f) dec[ep_rows[j]][f] = e.dec_host[j * 5 + f];
    } else {
      dec[ep_rows[j]][0] = e.amax_host[j];
    }
  }
}

// ----------------------------------------------------- native scheduler loop
// Restates continue_pipelined (pipeline.py:254-423), the executor's slot pool
// and metric counting (executor.py:76-107, 239-290) and greedy resolve
// (decisions.py:136-184). -1 stands for Python's None.
struct PLane {
  int stage = 0, index = 0, token = 0, state = -1, branch = 0, parent = -1, origin = -1;
  int first_token = -1, second_token = -1;
};

struct StatePool {
  std::priority_queue<int, std::vector<int>, std::greater<int>> free_;
  std::set<int> live_;
  explicit StatePool(int n) {
    for (int i = 0; i < n; ++i) free_.push(i);
  }
  int acquire() {
    REQUIRE(!free_.empty(), LS_ECAPACITY, "pipeline requires more recurrent state slots than configured");
    const int s = free_.top();
    free_.pop();
    live_.insert(s);
    return s;
  }
  void retain(const std::vector<PLane>& lanes) {
    std::set<int> keep;
    for (auto& l : lanes)
      if (l.state >= 0) keep.insert(l.state);
    for (auto it = live_.begin(); it != live_.end();) {
      if (!keep.count(*it)) {
        free_.push(*it);
        it = live_.erase(it);
      } else {
        ++it;
      }
    }
  }
};

bool descends_from(int b, int anc, const std::map<int, int>& parents) {
  while (b != -1 && b != anc) {
    auto it = parents.find(b);
    b = it == parents.end() ? -1 : it->second;
  }
  return b == anc;
}

std::map<int, int> prune_ancestry(const std::vector<PLane>& lanes, int root,
                                  const std::map<int, int>& parents) {
  std::set<int> live{root};
  for (auto& l : lanes) {
    int b = l.branch;
    while (b != root) {
      auto it = parents.find(b);
      REQUIRE(b != -1 && it != parents.end(), LS_EPIPELINE, "pipeline branch escaped the selected ancestry");
      live.insert(b);
      b = it->second;
    }
  }
  std::map<int, int> out;
  for (int b : live) out[b] = b == root ? -1 : parents.at(b);
  return out;
}

// What the scheduler loop needs from an executor besides the cycle itself:
// the schedule, how decisions are resolved, branch retention and the stop
// rule of one request. The engine binds retention to the request's GPU
// timelines; ls_pipeline_simulate binds it to a host callback so the same
// loop is testable without a GPU.
struct SchedHooks {
  int S = 0, K = 1, X = 0, max_rows = 0;
  bool sampling = false;   // decisions are sampled 5-field rows, else greedy argmax
  std::map<int, int> endpoint_kind;
  std::function<void(const std::vector<PLane>&, int accepted_stage)> retain;
  std::function<bool(const std::vector<long long>&)> should_stop;
};

// One request's pipeline (continue_pipelined, pipeline.py:254-423) as a state
// machine, so that the lanes of several requests can share each cycle:
// gather() adds this cycle's lanes, consume() takes their decisions and runs
// the loop body (resolve, commit, branch selection, pruning, retention).
struct PipelineRun {
  const SchedHooks& hk;
  int req, state_base, max_new;
  std::vector<long long> committed;
  ls_stats st{};
  StatePool pool;
  int next_branch = 1;
  std::map<int, int> parents{{0, -1}};
  std::vector<PLane> lanes;
  bool done = false;
  double* decode_t0;

  PipelineRun(const SchedHooks& h, int r, int base, long long first, int mx, double* t0)
      : hk(h), req(r), state_base(base), max_new(mx), committed{first}, pool(h.max_rows),
        decode_t0(t0) {
    if (stop() || max_new == 1) {
      hk.retain({}, -1);
      done = true;
      return;
    }
    lanes.resize(1);
    lanes[0].index = 1;
    lanes[0].token = (int)first;
  }

  bool stop() {
    if (*decode_t0 < 0) *decode_t0 = now_s();
    return hk.should_stop(committed);
  }

  // executor.forward's lanes: every live lane, with a state slot
  void gather(std::vector<CycleLane>& cl) {
    for (auto& l : lanes) {
      if (l.state < 0) l.state = pool.acquire();  // written back as result.state
      CycleLane c{l.stage, l.index, l.token, l.branch, l.parent, state_base + l.state};
      c.origin = l.origin;
      c.first = l.first_token;
      c.second = l.second_token;
      c.req = req;
      cl.push_back(c);
    }
  }

  // dec: this request's decisions, in gather() order
  void consume(const Dec* dec) {
    const int q1 = hk.K - 1, q2 = hk.X ? hk.K * hk.X - 1 : -1, final_stage = hk.S - 1;
    st.pipeline_cycles += 1;
    st.recurrent_rows += (int64_t)lanes.size() * hk.K;
    for (auto& l : lanes) {
      st.pre_rows += l.stage == 0;
      st.post_rows += hk.endpoint_kind.count(l.stage + hk.K - 1);
    }
    // continue_pipelined body
    std::vector<PLane> following, children;
    int final_idx = -1;
    long long final_pred = 0;
    int accepted_stage = -1;
    for (size_t i = 0; i < lanes.size(); ++i) {
      PLane& l = lanes[i];
      const int end_stage = l.stage + hk.K - 1;
      auto kit = hk.endpoint_kind.find(end_stage);
      const int kind = kit == hk.endpoint_kind.end() ? -1 : kit->second;
      // resolve (greedy: decisions.py:136-184; sampling: policy.py:285-308)
      const Dec& d = dec[i];
      const long long pred = d[0];
      bool proposed = false, fr = false, sr = false;
      int acc = -1;
      if (hk.sampling) {
        proposed = d[1] != 0;
        acc = d[2] == 1 ? q1 : d[2] == 2 ? q2 : -1;
        fr = d[3] != 0;
        sr = d[4] != 0;
      } else {
        proposed = kind == 0 || (kind == 1 && (l.first_token < 0 || pred != l.first_token));
        if (kind == 2 && l.first_token >= 0) {
          fr = pred != l.first_token;
          if (!fr) acc = q1;
          else if (l.second_token >= 0) {
            sr = pred != l.second_token;
            if (!sr) acc = q2;
          }
        }
      }
      if (end_stage == final_stage) {
        REQUIRE(final_idx < 0, LS_EPIPELINE, "multiple branches reached the final stage");
        final_idx = (int)i;
        final_pred = pred;
        accepted_stage = acc;
        // executor.py:268-281
        const bool sv = fr && l.second_token >= 0;
        st.verified_proposals += 1;
        st.first_rejections += fr;
        st.second_verifications += sv;
        st.second_acceptances += sv && acc == q2;
        st.second_rejections += sv && sr;
        continue;
      }
      l.stage = end_stage + 1;
      if ((end_stage == q1 || end_stage == q2) && kind >= 0 && proposed) {
        if (end_stage == q1) l.first_token = (int)pred;
        else l.second_token = (int)pred;
        if (l.index + 1 < max_new) {
          PLane c;
          c.stage = 0;
          c.index = l.index + 1;
          c.token = (int)pred;
          c.branch = next_branch;
          c.parent = l.branch;
          c.origin = end_stage;
          children.push_back(c);
          parents[next_branch] = l.branch;
          next_branch++;
        }
      }
      following.push_back(l);
    }
    following.insert(following.end(), children.begin(), children.end());
    if (final_idx >= 0) {
      const PLane fl = lanes[final_idx];
      REQUIRE(fl.index == (int)committed.size(), LS_EPIPELINE, "pipeline attempted to commit out of order");
      committed.push_back(final_pred);
      if (stop()) {
        lanes.clear();
        pool.retain(lanes);
        hk.retain({}, -1);
        done = true;
        return;
      }
      accepted_stage = fl.first_token >= 0 ? accepted_stage : -1;
      if (fl.index + 1 < max_new) {
        int sel = -1;
        for (size_t j = 0; j < following.size(); ++j) {
          const PLane& c = following[j];
          if (c.parent == fl.branch && c.token == final_pred && c.origin == accepted_stage &&
              accepted_stage >= 0) {
            sel = (int)j;
            break;
          }
        }
        int keep;
        if (sel < 0) {
          PLane c;
          c.stage = 0;
          c.index = fl.index + 1;
          c.token = (int)final_pred;
          c.branch = next_branch;
          c.parent = fl.branch;
          c.origin = final_stage;
          parents[next_branch] = fl.branch;
          next_branch++;
          following.push_back(c);
          keep = c.branch;
        } else {
          keep = following[sel].branch;
        }
        std::vector<PLane> kept;
        for (auto& c : following)
          if (descends_from(c.branch, keep, parents)) kept.push_back(c);
        following.swap(kept);
        parents = prune_ancestry(following, keep, parents);
      } else {
        following.clear();
        accepted_stage = -1;
      }
    }
    REQUIRE((int)following.size() <= hk.max_rows, LS_EPIPELINE, "speculative tree exceeded branch row limit");
    lanes.swap(following);
    pool.retain(lanes);
    hk.retain(lanes, accepted_stage);
    REQUIRE(!lanes.empty() || (int)committed.size() >= max_new, LS_EPIPELINE,
            "pipeline drained before generation completed");
    if ((int)committed.size() >= max_new) done = true;
  }
};

using Forward = std::function<void(const std::vector<CycleLane>&, std::vector<Dec>&)>;

// Run the pipelines of several requests until all are done, each cycle over
// the lanes of every request still running.
void drive(std::vector<std::unique_ptr<PipelineRun>>& runs, const Forward& forward) {
  std::vector<CycleLane> cl;
  std::vector<Dec> dec;
  std::vector<size_t> off(runs.size());
  for (;;) {
    cl.clear();
    for (size_t i = 0; i < runs.size(); ++i) {
      off[i] = cl.size();
      if (!runs[i]->done) runs[i]->gather(cl);
    }
    if (cl.empty()) return;
    forward(cl, dec);
    for (size_t i = 0; i < runs.size(); ++i)
      if (!runs[i]->done && off[i] < cl.size() && cl[off[i]].req == runs[i]->req)
        runs[i]->consume(dec.data() + off[i]);
  }
}

using StopRule = std::function<bool(const std::vector<long long>&)>;

// Stop after a commit when the caller's callback asks to (it sees the whole
// committed output, as the reference's should_stop does), or at the EOS id.
StopRule stop_rule(long long stop_token, ls_commit_fn fn, void* user) {
  return [stop_token, fn, user](const std::vector<long long>& ids) {
    static_assert(sizeof(long long) == sizeof(int64_t), "committed ids are passed as int64");
    if (fn && fn(user, reinterpret_cast<const int64_t*>(ids.data()), (int)ids.size()) != 0) return true;
    return stop_token >= 0 && ids.back() == stop_token;
  };
}

// Autoregressive decoding of several requests together (serving.py:216-239):
// per step one lane per running request through pre, S core iterations and
// post, each role as one call over all of them.
void run_ar(ls_engine& e, std::vector<std::vector<long long>>& committed, std::vector<int>& reqs,
            const std::vector<StopRule>& stop, int max_new, double& decode_t0) {
  const int n = (int)reqs.size();
  decode_t0 = now_s();
  std::vector<char> done(n, 0);
  for (int i = 0; i < n; ++i) done[i] = stop[i](committed[i]) || (int)committed[i].size() >= max_new;
  const bool pre_attn = e.mc.n_pre_layers > 0, post_attn = e.mc.n_post_layers > 0;
  std::vector<int> act, tok, pos, slot;
  std::vector<Cursor*> c;
  for (;;) {
    act.clear();
    for (int i = 0; i < n; ++i)
      if (!done[i]) act.push_back(i);
    if (act.empty()) break;
    const int B = (int)act.size();
    tok.assign(B, 0);
    pos.assign(B, 0);
    slot.assign(B, -1);
    c.assign(B, nullptr);
    for (int j = 0; j < B; ++j) {
      Request& R = e.reqs[reqs[act[j]]];
      tok[j] = (int)committed[act[j]].back();
      pos[j] = R.prefill_len + (int)committed[act[j]].size();   // index = tokens committed so far
    }
    auto role = [&](int r, int depth) {
      int* m = stage_meta(e);
      const bool attn = r == kCore || (r == kPre && pre_attn) || (r == kPost && post_attn);
      for (int j = 0; j < B; ++j) {
        Request& R = e.reqs[reqs[act[j]]];
        c[j] = attn ? R.tl.get_or_create_cursor(r, depth, 0, -1) : nullptr;
        slot[j] = fill_lane(e, R.tl, m, j, tok[j], pos[j], c[j], r == kPre ? -1 : R.state_base,
                            r == kPost ? -1 : R.state_base);
        if (r == kPost) set_final_readout(e, m, j, R, (int)(++R.draw_cycle), 0);
      }
      run_role(e, r, B, m, true);
      for (int j = 0; j < B; ++j)
        if (c[j]) advance(c[j], slot[j], true);
    };
    role(kPre, 0);
    for (int s = 0; s < e.S; ++s) role(kCore, s);
    role(kPost, e.S - 1);
    long long* src = e.sampling ? e.dec_dev : e.amax_dev;
    const int stride = e.sampling ? 5 : 1;
    CK(cudaMemcpyAsync(e.dec_host, src, sizeof(long long) * stride * B, cudaMemcpyDeviceToHost, e.stream));
    e.d2h_bytes += sizeof(long long) * stride * B;
    fetch_device_error(e);
    CK(cudaStreamSynchronize(e.stream));
    e.host_syncs++;
    e.staging_next = 0;
    check_fetched_error(e);
    for (int j = 0; j < B; ++j) {
      const int i = act[j];
      committed[i].push_back(e.dec_host[j * stride]);
      if (stop[i](committed[i]) || (int)committed[i].size() >= max_new) done[i] = 1;
    }
  }
  for (int i = 0; i < n; ++i) e.reqs[reqs[i]].tl.retain({});
}

// ------------------------------------------------ device-resident decode loop
// Where the scheduler kernels write the role calls' metadata (fixed width
// max_rows, unused lanes inactive).
LoopMeta loop_meta_of(const ls_engine& e) {
  const long F = (long)kMetaFields * e.cap;
  return LoopMeta{e.loop_meta, e.loop_meta + F, F, e.loop_meta + (1 + e.K) * F, e.max_rows, e.loop_active};
}

// `cycles` cycles as one graph. In each, the role calls read the metadata the
// previous scheduler kernel wrote (the post call's lm_head GEMM reduces each
// lane's greedy token, or the sampler writes its decision rows), then the
// step kernel resolves the decisions, commits, retains branches and plans the
// next cycle. Nothing returns to the host between cycles. Inside a graph, an
// Ouro cycle's first kernel (the embedding prep) is launched while the step
// kernel before it still runs, and reads the metadata after its PDL wait.
constexpr int kLoopGraphCycles = 8;
const ls_engine::LoopGraph& loop_graph_for(ls_engine& e, int chunks, int cycles) {
  const int key = (chunks * 2 + (e.sampling ? 1 : 0)) * (kLoopGraphCycles + 1) + cycles;
  auto it = e.loop_graphs.find(key);
  if (it != e.loop_graphs.end()) return it->second;
  const int W = e.max_rows;
  const LoopMeta lm = loop_meta_of(e);
  int* pre = lm.pre;
  int* core = lm.core;
  const long F = lm.stride;
  int* post = lm.post;
  int kernels = 0;
  const bool early_prep = e.mc.family == LS_FAMILY_OURO && e.sc.use_pdl != 0;
  CK(cudaStreamBeginCapture(e.stream, cudaStreamCaptureModeThreadLocal));
  try {
    for (int cyc = 0; cyc < cycles; ++cyc) {
      e.qkv_planes = true;    // one new position per lane
      e.attn_chunks = chunks;
      // the first role kernel reads the metadata the step kernel wrote
      if (cyc > 0 && early_prep) e.meta_after_wait = 1;
      else e.serialize_next = true;
      // the attention form is chosen for the full width, so that a cycle whose
      // lanes are all live still runs its attention in one wave (every form
      // computes the same values)
      e.attn_form_lanes = W;
      e.meta_override = pre;
      e.gemm_active = lm.active;
      enqueue_role(e, kPre, W);
      kernels += e.kernels_in_call;
      e.gemm_active = lm.active + 1;
      for (int k = 0; k < e.K; ++k) {
        e.meta_override = core + k * F;
        enqueue_role(e, kCore, W);
        kernels += e.kernels_in_call;
      }
      e.meta_override = post;
      e.gemm_active = lm.active + 2;
      enqueue_role(e, kPost, W);
      kernels += e.kernels_in_call;
      e.meta_override = nullptr;
      e.gemm_active = nullptr;
      const bool pdl = e.sc.use_pdl != 0;
      if (e.sampling)
        launch(loop_step_kernel, dim3(1), dim3(kLoopThreads), 0, e.stream, pdl, e.loop_sched,
               (const long long*)e.dec_dev, 5, e.loop_out, lm);
      else
        launch(loop_step_kernel, dim3(1), dim3(kLoopThreads), 0, e.stream, pdl, e.loop_sched,
               (const long long*)e.amax_dev, 1, e.loop_out, lm);
      kernels += 1;
    }
  } catch (...) {
    e.meta_override = nullptr;
    e.gemm_active = nullptr;
    e.meta_after_wait = 0;
    e.attn_form_lanes = 0;
    cudaGraph_t g = nullptr;
    cudaStreamEndCapture(e.stream, &g);
    if (g) cudaGraphDestroy(g);
    throw;
  }
  e.attn_form_lanes = 0;
  cudaGraph_t g = nullptr;
  CK(cudaStreamEndCapture(e.stream, &g));
  ls_engine::LoopGraph lg;
  const cudaError_t ie = cudaGraphInstantiate(&lg.exec, g, 0);
  cudaGraphDestroy(g);
  CK(ie);
  lg.kernels = kernels;
  return e.loop_graphs.emplace(key, lg).first->second;
}

const char* loop_error_text(int code) {
  static const char* names[] = {"ok", "recurrent state slots exhausted", "mapping rows exhausted",
                                "KV slots exhausted", "branch with an unavailable parent",
                                "several lanes reached the final stage", "commit out of order",
                                "speculative tree exceeded the branch row limit",
                                "pipeline drained before generation completed", "scheduler table full"};
  return code > 0 && code < 10 ? names[code] : "unknown";
}

// One request on the device-resident loop, after its prefill. A cycle commits
// at most one token, so the host launches a batch of at most as many cycles as
// tokens remain (64; 16 when an EOS id may end the request early, which
// bounds the cycles run after it), then reads the scheduler state, and
// repeats until the request is done. Each batch uses the graph whose
// attention grid covers the longest timeline the batch can reach: no lane is
// more than S positions ahead of the committed tokens.
std::vector<long long> run_device_loop(ls_engine& e, Request& R, long long first, int max_new,
                                       long long stop_token, ls_stats& st, double& decode_t0) {
  LoopSched& h = *e.loop_host;
  std::memset(&h, 0, sizeof(LoopSched));
  long long first_out = 0;
  ds_start(h, e.S, e.K, e.X, e.max_rows, max_new, stop_token, first, &first_out);
  h.has_pre = e.mc.n_pre_layers > 0;
  h.has_post = e.mc.n_post_layers > 0;
  h.prefill_len = R.prefill_len;
  h.state_base = R.state_base;
  h.draw_cycle = (int)R.draw_cycle;
  h.seed = R.seed;
  R.tl.export_to(h);
  decode_t0 = now_s();
  std::vector<long long> ids{first};
  if (h.done) return ids;
  CK(cudaMemcpyAsync(e.loop_sched, &h, sizeof(LoopSched), cudaMemcpyHostToDevice, e.stream));
  CK(cudaMemcpyAsync(e.loop_out, &first_out, sizeof(long long), cudaMemcpyHostToDevice, e.stream));
  e.h2d_bytes += sizeof(LoopSched) + sizeof(long long);
  launch(loop_plan_kernel, dim3(1), dim3(kLoopThreads), 0, e.stream, false, e.loop_sched, loop_meta_of(e));
  e.kernel_launches += 1;
  long cycles = 0;
  int committed = 1;
  const int batch_max = stop_token >= 0 ? 16 : 64;
  for (;;) {
    const int nb = std::min(max_new - committed, batch_max);
    int chunks = cdiv(R.prefill_len + committed + nb + e.S + 1, kAttnChunk);
    chunks = std::min(chunks + (chunks & 1), e.max_chunks);
    const ls_engine::LoopGraph& lg = loop_graph_for(e, chunks, kLoopGraphCycles);
    for (int i = 0; i < nb / kLoopGraphCycles; ++i) CK(cudaGraphLaunch(lg.exec, e.stream));
    e.kernel_launches += (long)(nb / kLoopGraphCycles) * lg.kernels;
    if (nb % kLoopGraphCycles) {
      const ls_engine::LoopGraph& l1 = loop_graph_for(e, chunks, 1);
      for (int i = 0; i < nb % kLoopGraphCycles; ++i) CK(cudaGraphLaunch(l1.exec, e.stream));
      e.kernel_launches += (long)(nb % kLoopGraphCycles) * l1.kernels;
    }
    cycles += nb;
    CK(cudaMemcpyAsync(&h, e.loop_sched, sizeof(LoopSched), cudaMemcpyDeviceToHost, e.stream));
    e.d2h_bytes += sizeof(LoopSched);
    fetch_device_error(e);
    CK(cudaStreamSynchronize(e.stream));
    e.host_syncs++;
    check_fetched_error(e);
    REQUIRE(h.err == kDsOk, LS_EPIPELINE, std::string("device loop: ") + loop_error_text(h.err));
    committed = h.committed;
    if (h.done || committed >= max_new) break;
  }
  ids.resize(h.committed);
  CK(cudaMemcpy(ids.data(), e.loop_out, sizeof(long long) * h.committed, cudaMemcpyDeviceToHost));
  e.d2h_bytes += sizeof(long long) * h.committed;
  st.pipeline_cycles = h.stats[0];
  st.pre_rows = h.stats[1];
  st.recurrent_rows = h.stats[2];
  st.post_rows = h.stats[3];
  st.verified_proposals = h.stats[4];
  st.first_rejections = h.stats[5];
  st.second_verifications = h.stats[6];
  st.second_acceptances = h.stats[7];
  st.second_rejections = h.stats[8];
  // every launched cycle streams the weights of all its role calls
  e.core_calls += cycles * e.K;
  e.post_calls += cycles;
  if (e.mc.n_pre_layers > 0) e.pre_calls += cycles;
  e.core_kv_positions += h.kv_positions;
  R.draw_cycle = (uint32_t)h.draw_cycle;
  return ids;
}

SchedHooks engine_hooks(ls_engine& e, int req, StopRule stop) {
  SchedHooks hk;
  hk.S = e.S;
  hk.K = e.K;
  hk.X = e.X;
  hk.max_rows = e.max_rows;
  hk.endpoint_kind = e.endpoint_kind;
  hk.sampling = e.reqs[req].sampled;
  hk.retain = [&e, req](const std::vector<PLane>& lanes, int) {
    std::vector<std::pair<int, int>> bp;
    for (auto& l : lanes) bp.emplace_back(l.branch, l.parent);
    e.reqs[req].tl.retain(bp);
  };
  hk.should_stop = std::move(stop);
  return hk;
}

int fail(ls_engine* e, const std::exception& ex) {
  const EngineError* ee = dynamic_cast<const EngineError*>(&ex);
  if (e) e->last_error = ex.what();
  else g_last_error = ex.what();
  return ee ? ee->code : LS_EINVAL;
}

}  // namespace

// ================================================ standalone decode attention
namespace {

int fail_global(const std::exception& ex) {
  const EngineError* ee = dynamic_cast<const EngineError*>(&ex);
  g_last_error = ex.what();
  return ee ? ee->code : LS_EINVAL;
}

// Scratch of one decode-attention call, carved from a byte buffer: an error
// word, the per-chunk partials (acc, then max/sum) and the arrival tickets.
struct AttnScratch {
  int* err;
  float* o_part;
  float* ml_part;
  int* tickets;
  size_t ticket_bytes;
  size_t total;
};

AttnScratch carve_attn_scratch(char* base, int n, int nh, int nkv, int hd, int max_chunks) {
  AttnScratch s{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    char* p = base ? base + off : nullptr;
    off += (bytes + 255) / 256 * 256;
    return p;
  };
  s.err = reinterpret_cast<int*>(take(sizeof(int)));
  s.o_part = reinterpret_cast<float*>(take(sizeof(float) * (size_t)n * nh * max_chunks * hd));
  s.ml_part = reinterpret_cast<float*>(take(sizeof(float) * (size_t)n * nh * max_chunks * 2));
  s.ticket_bytes = sizeof(int) * (size_t)n * nkv;
  s.tickets = reinterpret_cast<int*>(take(s.ticket_bytes));
  s.total = off;
  return s;
}

void check_attn_shape(int n, int nh, int nkv, int hd, int n_slots, int n_rows, int max_ctx) {
  REQUIRE(n >= 1 && nh >= 1 && nkv >= 1 && n_slots >= 1 && n_rows >= 1, LS_EINVAL,
          "decode attention: sizes must be positive");
  REQUIRE(nh % nkv == 0, LS_EINVAL, "decode attention: n_heads must be a multiple of n_kv_heads");
  const int G = nh / nkv;
  REQUIRE((hd == 64 && (G == 1 || G == 2 || G == 4)) || (hd == 128 && (G == 1 || G == 2)),
          LS_EINVAL, "decode attention: unsupported head_dim / GQA group");
  REQUIRE(max_ctx >= 1 && cdiv(max_ctx, kAttnChunk) <= kAttnMaxChunks, LS_EINVAL,
          "decode attention: max_context must be in [1, 131072]");
}

// Launch one decode-attention call on `stream` using `sc` as scratch, wait
// for it, and report a device-side index error as LS_EDEVICE.
void run_decode_attention(const float* q, const void* k_pool, const void* v_pool, const int32_t* map,
                          const int32_t* lane_rows, const int32_t* lane_lens, int n, int nh, int nkv,
                          int hd, int n_slots, int n_rows, int max_ctx, const AttnScratch& sc,
                          float* out, cudaStream_t stream) {
  const int max_chunks = cdiv(max_ctx, kAttnChunk);
  CK(cudaMemsetAsync(sc.err, 0, sizeof(int), stream));
  CK(cudaMemsetAsync(sc.tickets, 0, sc.ticket_bytes, stream));   // tickets start at zero
  AttnArgs a{Meta{nullptr, 0}, nh, nkv, q, map, max_ctx, n_rows,
             static_cast<const bf16*>(k_pool), static_cast<const bf16*>(v_pool), n_slots,
             max_chunks, sc.o_part, sc.ml_part, sc.tickets, nullptr, out, lane_lens, lane_rows,
             1.0f / std::sqrt((float)hd), sc.err};
  const dim3 grid(n, nkv, max_chunks), blk(kAttnThreads);
  const int G = nh / nkv;
  int dev = 0, sms = 148;
  CK(cudaGetDevice(&dev));
  CK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const int form = attention_form((long)n * nkv * max_chunks, sms);
#define LS_ATTN(HD_, G_)                                                                        \
  (form == kAttnWide  ? launch(attn_kernel<HD_, G_, kAttnWide>, grid, blk, 0, stream, false, a)  \
   : form == kAttnMid ? launch(attn_kernel<HD_, G_, kAttnMid>, grid, blk, 0, stream, false, a)   \
                      : launch(attn_kernel<HD_, G_, kAttnVLate>, grid, blk, 0, stream, false, a))
  if (hd == 128 && G == 1) LS_ATTN(128, 1);
  else if (hd == 128 && G == 2) LS_ATTN(128, 2);
  else if (hd == 64 && G == 1) LS_ATTN(64, 1);
  else if (hd == 64 && G == 2) LS_ATTN(64, 2);
  else LS_ATTN(64, 4);
#undef LS_ATTN
  int err = 0;
  CK(cudaMemcpyAsync(&err, sc.err, sizeof(int), cudaMemcpyDeviceToHost, stream));
  CK(cudaStreamSynchronize(stream));
  REQUIRE(err == kDevOk, LS_EDEVICE, "decode attention: a lane row, length or KV slot was out of range");
}

// ---------------------------------------------- allocation-free variant
// Some callers cannot call cudaMalloc: code running inside an allocator or
// memory-pool hook, a runtime whose device memory is fully reserved up front,
// or a process that forbids device allocation after start-up. For them the
// decode attention can use this fixed scratch instead of a caller workspace.
// Every GPU that loads the library holds these bytes until the process exits,
// and every call on a device shares them: the last call's contents stay there
// (the call clears its error word and arrival tickets itself), and calls
// that overlap on the GPU race on it.
constexpr size_t kNoAllocScratchBytes = 4u << 20;   // 4 MiB
static __device__ __align__(256) char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mutex;
char* g_noalloc_ptr[kMaxDevices] = {};

// Device address of the scratch array on the current device. In host code
// the array's name is only a host-side stand-in, so the real address is
// looked up once per device (the first call on that device does it, with
// that device current) and cached for the life of the process: the cache
// assumes the device is not reset (cudaDeviceReset) while the library is
// loaded.
char* noalloc_scratch_for_current_device() {
  int dev = -1;
  CK(cudaGetDevice(&dev));
  REQUIRE(dev >= 0 && dev < kMaxDevices, LS_EINVAL, "device ordinal out of range");
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    CK(cudaGetSymbolAddress(&p, g_noalloc_scratch));
    REQUIRE(p != nullptr, LS_ECUDA, "cudaGetSymbolAddress returned no address");
    g_noalloc_ptr[dev] = static_cast<char*>(p);
  }
  return g_noalloc_ptr[dev];
}

}  // namespace

// ======================================================================== C ABI
extern "C" {

int ls_decode_attention_noalloc(const float* q, const void* k_pool, const void* v_pool,
                                const int32_t* map, const int32_t* lane_rows,
                                const int32_t* lane_lens, int n_lanes, int n_heads, int n_kv_heads,
                                int head_dim, int n_slots, int n_rows, int max_context, float* out,
                                void* stream) {
  if (!q || !k_pool || !v_pool || !map || !lane_rows || !lane_lens || !out) {
    g_last_error = "decode attention (no-alloc): null pointer argument";
    return LS_EINVAL;
  }
  try {
    check_attn_shape(n_lanes, n_heads, n_kv_heads, head_dim, n_slots, n_rows, max_context);
    const int max_chunks = cdiv(max_context, kAttnChunk);
    const size_t need =
        carve_attn_scratch(nullptr, n_lanes, n_heads, n_kv_heads, head_dim, max_chunks).total;
    REQUIRE(need <= kNoAllocScratchBytes, LS_ECAPACITY,
            "decode attention (no-alloc): this shape needs " + std::to_string(need) +
                " scratch bytes, above the fixed " + std::to_string(kNoAllocScratchBytes) +
                " (lanes x heads x ceil(max_context/128) x (head_dim + 2) x 4 bytes must fit); "
                "use ls_decode_attention with a workspace");
    char* base = noalloc_scratch_for_current_device();
    const AttnScratch sc =
        carve_attn_scratch(base, n_lanes, n_heads, n_kv_heads, head_dim, max_chunks);
    run_decode_attention(q, k_pool, v_pool, map, lane_rows, lane_lens, n_lanes, n_heads, n_kv_heads,
                         head_dim, n_slots, n_rows, max_context, sc, out,
                         static_cast<cudaStream_t>(stream));
  } catch (const std::exception& ex) {
    return fail_global(ex);
  }
  return LS_OK;
}

size_t ls_decode_attention_noalloc_limit(void) { return kNoAllocScratchBytes; }


size_t ls_decode_attention_workspace_bytes(int n_lanes, int n_heads, int n_kv_heads, int head_dim,
                                           int max_context) {
  if (n_lanes < 1 || n_heads < 1 || n_kv_heads < 1 || head_dim < 1 || max_context < 1) return 0;
  return carve_attn_scratch(nullptr, n_lanes, n_heads, n_kv_heads, head_dim,
                            cdiv(max_context, kAttnChunk)).total;
}

int ls_decode_attention(const float* q, const void* k_pool, const void* v_pool, const int32_t* map,
                        const int32_t* lane_rows, const int32_t* lane_lens, int n_lanes, int n_heads,
                        int n_kv_heads, int head_dim, int n_slots, int n_rows, int max_context,
                        void* workspace, size_t workspace_bytes, float* out, void* stream) {
  if (!q || !k_pool || !v_pool || !map || !lane_rows || !lane_lens || !workspace || !out) {
    g_last_error = "decode attention: null pointer argument";
    return LS_EINVAL;
  }
  try {
    check_attn_shape(n_lanes, n_heads, n_kv_heads, head_dim, n_slots, n_rows, max_context);
    const AttnScratch sc = carve_attn_scratch(static_cast<char*>(workspace), n_lanes, n_heads,
                                              n_kv_heads, head_dim, cdiv(max_context, kAttnChunk));
    REQUIRE(workspace_bytes >= sc.total, LS_EINVAL,
            "decode attention: workspace smaller than ls_decode_attention_workspace_bytes()");
    REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 255) == 0, LS_EINVAL,
            "decode attention: workspace must be 256-byte aligned");
    run_decode_attention(q, k_pool, v_pool, map, lane_rows, lane_lens, n_lanes, n_heads, n_kv_heads,
                         head_dim, n_slots, n_rows, max_context, sc, out,
                         static_cast<cudaStream_t>(stream));
  } catch (const std::exception& ex) {
    return fail_global(ex);
  }
  return LS_OK;
}


const char* ls_version(void) { return "loopspec-b200 0.1.0 (sm_100a)"; }

const char* ls_last_error(ls_engine* e) { return e ? e->last_error.c_str() : g_last_error.c_str(); }

int ls_create(const ls_model_cfg* model, const ls_sched_cfg* sched, int device, ls_engine** out) {
  if (!model || !sched || !out) return LS_EINVAL;
  *out = nullptr;
  std::unique_ptr<ls_engine> e(new ls_engine());
  try {
    e->mc = *model;
    e->sc = *sched;
    e->device = device;
    REQUIRE(model->family == LS_FAMILY_OURO || model->family == LS_FAMILY_RAVEN, LS_EINVAL, "bad family");
    REQUIRE(model->layout >= 0 && model->layout <= 2, LS_EINVAL, "bad layout");
    REQUIRE((model->family == LS_FAMILY_OURO) == (model->layout == LS_LAYOUT_OURO), LS_EINVAL,
            "Ouro uses the ouro layout; Raven uses raven_pre or olmo_post");
    REQUIRE(model->stages > 0, LS_EINVAL, "stages S must be a positive integer");
    // PipelineSchedule.__post_init__ (pipeline.py:132-139)
    const int S = model->stages, K = sched->step_size, X = sched->second_step;
    REQUIRE(K >= 1 && K < S && S % K == 0, LS_EINVAL,
            "step_size K must be a positive divisor of S with K < S");
    REQUIRE(X == 0 || (X > 1 && X < S / K), LS_EINVAL, "second_step X must satisfy 1 < X < S/K");
    e->S = S;
    e->K = K;
    e->X = X;
    e->depth = S / K;
    e->endpoint_kind[K - 1] = 0;
    if (X) e->endpoint_kind[K * X - 1] = 1;
    e->endpoint_kind[S - 1] = 2;
    long rows = 0;
    for (long b : e->birth_sizes()) rows += b;
    e->max_rows = (int)rows;
    CK(cudaSetDevice(device));
  } catch (const std::exception& ex) {
    return fail(nullptr, ex);
  }
  *out = e.release();
  return LS_OK;
}

int ls_load_weight(ls_engine* e, const char* name, const void* dptr, int dtype, const int64_t* shape,
                   int ndim) {
  if (!e || !name || !dptr || !shape || ndim < 1 || ndim > 4) return LS_EINVAL;
  try {
    REQUIRE(!e->finalized, LS_EINVAL, "weights must be loaded before ls_finalize");
    REQUIRE(dtype == 0, LS_EINVAL, "only bf16 weights are accepted");
    REQUIRE((reinterpret_cast<uintptr_t>(dptr) & 15) == 0, LS_EINVAL, "weight pointer must be 16-byte aligned");
    e->weights[name] = {static_cast<const bf16*>(dptr), std::vector<int64_t>(shape, shape + ndim)};
  } catch (const std::exception& ex) {
    return fail(e, ex);
  }
  return LS_OK;
}

int ls_finalize(ls_engine* e) {
  if (!e) return LS_EINVAL;
  try {
    e->finalize();
  } catch (const std::exception& ex) {
    return fail(e, ex);
  }
  return LS_OK;
}

int ls_tp_init(ls_engine* e, int rank, int ranks, void* handle_out) {
  if (!e || !handle_out) return LS_EINVAL;
  try {
    REQUIRE(e->finalized, LS_EINVAL, "engine not finalized");
    REQUIRE(e->tp_region == nullptr, LS_EINVAL, "tensor parallelism already initialised");
    REQUIRE(ranks >= 2 && ranks <= kTpMax && rank >= 0 && rank < ranks, LS_EINVAL,
            "tensor parallelism needs 2..8 ranks and 0 <= rank < ranks");
    REQUIRE(e->graphs.empty(), LS_EINVAL, "initialise tensor parallelism before the first role call");
    CK(cudaSetDevice(e->device));
    // planes of the widest O / down projection of any stack
    int so = 1, sd = 1;
    for (const Stack* st : {&e->pre, &e->core, &e->post})
      for (const LayerW& w : st->layers) {
        so = std::max(so, w.g_o.splits);
        sd = std::max(sd, w.g_down.splits);
      }
    auto up = [](size_t b) { return (b + 255) & ~size_t(255); };
    e->tp_off_o = 256;
    e->tp_off_d = e->tp_off_o + up(sizeof(float) * (size_t)so * e->cap * e->H);
    e->tp_off_qk = e->tp_off_d + up(sizeof(float) * (size_t)sd * e->cap * e->H);
    e->tp_bytes = e->tp_off_qk + up(sizeof(float) * 2 * (size_t)e->cap);
    e->tp_region = e->dalloc<char>(e->tp_bytes);   // zeroed: flags and epoch start at 0
    cudaIpcMemHandle_t h;
    CK(cudaIpcGetMemHandle(&h, e->tp_region));
    unsigned char* out = static_cast<unsigned char*>(handle_out);
    std::memset(out, 0, LS_TP_HANDLE_BYTES);
    std::memcpy(out, &h, sizeof(h));
    CK(cudaDeviceGetPCIBusId(reinterpret_cast<char*>(out) + sizeof(h), LS_TP_HANDLE_BYTES - (int)sizeof(h) - 8,
                             e->device));
    std::memcpy(out + LS_TP_HANDLE_BYTES - 8, &e->tp_bytes, 8);
    e->tp_rank = rank;
    e->tp_want = ranks;
  } catch (const std::exception& ex) {
    return fail(e, ex);
  }
  return LS_OK;
}

int ls_tp_attach(ls_engine* e, const void* handles) {
  if (!e || !handles) return LS_EINVAL;
  try {
    REQUIRE(e->tp_region != nullptr && e->tp_ranks == 1, LS_EINVAL, "call ls_tp_init once, then ls_tp_attach once");
    CK(cudaSetDevice(e->device));
    const unsigned char* in = static_cast<const unsigned char*>(handles);
    const int n = e->tp_want;
    const int bus_len = LS_TP_HANDLE_BYTES - (int)sizeof(cudaIpcMemHandle_t) - 8;
    std::vector<std::string> bus(n);
    for (int r = 0; r < n; ++r) {
      const char* b = reinterpret_cast<const char*>(in + (size_t)r * LS_TP_HANDLE_BYTES + sizeof(cudaIpcMemHandle_t));
      bus[r] = std::string(b, strnlen(b, bus_len));
      size_t bytes = 0;
      std::memcpy(&bytes, in + (size_t)(r + 1) * LS_TP_HANDLE_BYTES - 8, 8);
      REQUIRE(bytes == e->tp_bytes, LS_EINVAL, "tensor-parallel ranks disagree on the exchange layout");
      for (int q = 0; q < r; ++q)
        // ranks wait on one another inside kernels, so each needs its own GPU
        REQUIRE(bus[q] != bus[r], LS_EINVAL, "two tensor-parallel ranks share one GPU");
    }
    std::vector<char*> base(n, nullptr);
    for (int r = 0; r < n; ++r) {
      if (r == e->tp_rank) {
        base[r] = e->tp_region;
        continue;
      }
      cudaIpcMemHandle_t h;
      std::memcpy(&h, in + (size_t)r * LS_TP_HANDLE_BYTES, sizeof(h));
      void* p = nullptr;
      CK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
      e->tp_opened.push_back(p);
      base[r] = static_cast<char*>(p);
    }
    e->tp_base = base;
    e->tp_ranks = n;
  } catch (const std::exception& ex) {
    return fail(e, ex);
  }
  return LS_OK;
}

int ls_debug_tp_silent_peer(ls_engine* e, int wait_ms) {
  if (!e) return LS_EINVAL;
  try {
    REQUIRE(e->tp_region != nullptr && e->tp_ranks == 1 && e->tp_want == 2, LS_EINVAL,
            "call ls_tp_init with 2 ranks first, and no ls_tp_attach");
    REQUIRE(wait_ms >= 1 && wait_ms <= 10000, LS_EINVAL, "wait limit must be 1..10000 ms");
    CK(cudaSetDevice(e->device));
    // a zeroed region of this GPU stands in for the peer: its flags never rise
    char* silent = e->dalloc<char>(e->tp_bytes);
    e->tp_base.assign(2, nullptr);
    e->tp_base[e->tp_rank] = e->tp_region;
    e->tp_base[1 - e->tp_rank] = silent;
    e->tp_wait_ns = 1000000ull * (unsigned long long)wait_ms;
    e->tp_ranks = 2;
  } catch (const std::exception& ex) {
    return fail(e, ex);
  }
  return LS_OK;
}

int ls_set_sampling(ls_engine* e, float temperature, int top_k, float top_p, uint64_t seed) {
  if (!e) return LS_EINVAL;
  try {
    REQUIRE(e->finalized, LS_EINVAL, "engine not finalized");
    REQUIRE(temperature >= 0.f && top_k >= 0 && top_p > 0.f && top_p <= 1.f, LS_EINVAL,
            "sampling needs temperature >= 0, top_k >= 0, 0 < top_p <= 1");
    e->sparams = sample_params(temperature, top_k, top_p, seed);
    e->sampling = params_sampled(e->sparams);
    CK(cudaStreamSynchronize(e->stream));
    for (int i = 0; i < e->max_req; ++i)
      CK(cudaMemcpy(e->sparams_dev + i, &e->sparams, sizeof(SampleParams), cudaMemcpyHostToDevice));
  } catch (const std::exception& ex) {
    return fail(e, ex);
  }
  return LS_OK;
}

int ls_prefill(ls_engine* e, const int64_t* prompt, int n, float* out_logits, int64_t* first) {
  if (!e || !prompt || !first) return LS_EINVAL;
  try {
    REQUIRE(e->finalized, LS_EINVAL, "engine not finalized");
    e->reqs[0].seed = e->sparams.seed;
    e->reqs[0].sampled = e->sampling;
    *first = prefill(*e, e->reqs[0], prompt, n, out_logits);
  } catch (const std::exception& ex) {
    return fail(e, ex);
  }
  return LS_OK;
}

int ls_cycle(ls_engine* e, const int64_t* lanes, int n, int64_t* out_dec, float* out_logits) {
  if (!e || !lanes || !out_dec || n < 1) return LS_EINVAL;
  try {
    REQUIRE(e->finalized, LS_EINVAL, "engine not finalized");
    CK(cudaSetDevice(e->device));
    std::vector<CycleLane> cl(n);
    for (int i = 0; i < n; ++i) {
      const int64_t* l = lanes + 8 * i;
      cl[i] = CycleLane{(int)l[0], (int)l[1], (int)l[2], (int)l[3], (int)l[4], (int)l[5]};
      cl[i].first = (int)l[6];
      cl[i].second = (int)l[7];
    }
    std::vector<Dec> dec;
    cycle(*e, cl, dec, out_logits);
    for (int i = 0; i < n; ++i)
      for (int f = 0; f < 5; ++f) out_dec[i * 5 + f] = dec[i][f];
  } catch (const std::exception& ex) {
    return fail(e, ex);
  }
  return LS_OK;
}

int ls_retain(ls_engine* e, const int64_t* branch_ids, const int64_t* parent_ids, int n) {
  if (!e || n < 0 || (n > 0 && (!branch_ids || !parent_ids))) return LS_EINVAL;
  try {
    REQUIRE(e->finalized, LS_EINVAL, "engine not finalized");
    std::vector<std::pair<int, int>> bp;
    for (int i = 0; i < n; ++i) bp.emplace_back((int)branch_ids[i], (int)parent_ids[i]);
    e->reqs[0].tl.retain(bp);
  } catch (const std::exception& ex) {
    return fail(e, ex);
  }
  return LS_OK;
}

namespace {
// Prefill each request in turn, then decode all of them together (LoopSpec:
// one pipeline per request, each cycle over every running request's lanes;
// AR: one lane per running request per step). per_request[i] receives
// request i's scheduler counters and tokens; total (optional) the sums plus
// the batch's work counters, copy volumes and decode timing.
int generate_batch(ls_engine* e, const int64_t* prompts, const int32_t* lens, int n_req, int max_new,
                   int mode, const std::vector<StopRule>& stop, const uint64_t* seeds,
                   int64_t* out_ids, int32_t* n_out, ls_stats* per_request, ls_stats* total,
                   long long device_loop_stop = -2, const SampleParams* params = nullptr) {
  if (!e || !prompts || !lens || !out_ids || !n_out || n_req < 1 || max_new < 1 ||
      (mode != 0 && mode != 1) || (int)stop.size() != n_req)
    return LS_EINVAL;
  try {
    REQUIRE(e->finalized, LS_EINVAL, "engine not finalized");
    REQUIRE(n_req <= e->max_req, LS_ECAPACITY,
            "more requests than the engine's max_requests (" + std::to_string(e->max_req) + ")");
    e->h2d_bytes = e->d2h_bytes = 0;
    // per-request parameters (else the engine's for every request): slot i
    // holds request i's; the post calls run the sampler when any request
    // samples (greedy rows of it take the argmax); restored afterwards
    struct ParamScope {
      ls_engine* e;
      bool active, saved;
      ~ParamScope() {
        if (!active) return;
        e->sampling = saved;
        cudaStreamSynchronize(e->stream);
        for (int i = 0; i < e->max_req; ++i)
          cudaMemcpy(e->sparams_dev + i, &e->sparams, sizeof(SampleParams), cudaMemcpyHostToDevice);
      }
    } scope{e, params != nullptr, e->sampling};
    if (params) {
      bool any = false;
      CK(cudaStreamSynchronize(e->stream));
      for (int i = 0; i < n_req; ++i) {
        any = any || params_sampled(params[i]);
        CK(cudaMemcpy(e->sparams_dev + i, &params[i], sizeof(SampleParams), cudaMemcpyHostToDevice));
      }
      e->sampling = any;
    }
    ls_stats tot{};
    std::vector<long long> first(n_req);
    long off = 0;
    for (int i = 0; i < n_req; ++i) {
      Request& R = e->reqs[i];
      R.sampled = params ? params_sampled(params[i]) : e->sampling;
      R.seed = seeds ? seeds[i] : e->sparams.seed + (unsigned long long)i;
      first[i] = prefill(*e, R, prompts + off, lens[i], nullptr);
      off += lens[i];
      float pms = 0.f;
      CK(cudaEventElapsedTime(&pms, e->ev0, e->ev1));
      tot.prefill_device_ms += pms;
      REQUIRE(R.prefill_len + max_new < e->max_ctx, LS_ECAPACITY,
              "prompt + max_new_tokens exceeds max_context");
    }
    double t0 = -1.0;
    const int64_t launches0 = e->kernel_launches;
    const int64_t pre0 = e->pre_calls, core0 = e->core_calls, kv0 = e->core_kv_positions,
                  post0 = e->post_calls, sync0 = e->host_syncs;
    CK(cudaEventRecord(e->ev0, e->stream));
    std::vector<std::vector<long long>> ids(n_req);
    std::vector<ls_stats> st(n_req, ls_stats{});
    // a single LoopSpec request whose stop rule is only the EOS id
    // (device_loop_stop >= -1) runs on the device-resident loop
    const bool on_device = mode == 0 && n_req == 1 && device_loop_stop >= -1 && e->loop_enabled &&
                           e->tp_ranks == 1;
    if (on_device) {
      ids[0] = run_device_loop(*e, e->reqs[0], first[0], max_new, device_loop_stop, st[0], t0);
    } else if (mode == 0) {
      std::vector<SchedHooks> hooks;
      hooks.reserve(n_req);
      for (int i = 0; i < n_req; ++i) hooks.push_back(engine_hooks(*e, i, stop[i]));
      std::vector<std::unique_ptr<PipelineRun>> runs;
      for (int i = 0; i < n_req; ++i)
        runs.emplace_back(new PipelineRun(hooks[i], i, e->reqs[i].state_base, first[i], max_new, &t0));
      drive(runs, [e](const std::vector<CycleLane>& cl, std::vector<Dec>& dec) { cycle(*e, cl, dec, nullptr); });
      for (int i = 0; i < n_req; ++i) {
        ids[i] = runs[i]->committed;
        st[i] = runs[i]->st;
      }
    } else {
      std::vector<int> reqs(n_req);
      for (int i = 0; i < n_req; ++i) {
        reqs[i] = i;
        ids[i] = {first[i]};
      }
      run_ar(*e, ids, reqs, stop, max_new, t0);
    }
    CK(cudaEventRecord(e->ev1, e->stream));
    CK(cudaEventSynchronize(e->ev1));
    const double t1 = now_s();
    float dms = 0.f;
    CK(cudaEventElapsedTime(&dms, e->ev0, e->ev1));
    for (int i = 0; i < n_req; ++i) {
      st[i].decode_tokens = std::max<int64_t>((int64_t)ids[i].size() - 1, 0);
      st[i].decode_device_ms = dms;
      st[i].decode_host_s = t0 >= 0 ? t1 - t0 : 0.0;
      for (size_t k = 0; k < ids[i].size(); ++k) out_ids[(long)i * max_new + k] = ids[i][k];
      n_out[i] = (int32_t)ids[i].size();
      if (per_request) per_request[i] = st[i];
      tot.pipeline_cycles += st[i].pipeline_cycles;
      tot.pre_rows += st[i].pre_rows;
      tot.recurrent_rows += st[i].recurrent_rows;
      tot.post_rows += st[i].post_rows;
      tot.verified_proposals += st[i].verified_proposals;
      tot.first_rejections += st[i].first_rejections;
      tot.second_verifications += st[i].second_verifications;
      tot.second_acceptances += st[i].second_acceptances;
      tot.second_rejections += st[i].second_rejections;
      tot.decode_tokens += st[i].decode_tokens;
    }
    tot.decode_device_ms = dms;
    tot.decode_host_s = t0 >= 0 ? t1 - t0 : 0.0;
    tot.h2d_bytes = e->h2d_bytes;
    tot.d2h_bytes = e->d2h_bytes;
    tot.decode_kernel_launches = e->kernel_launches - launches0;
    tot.pre_calls = e->pre_calls - pre0;
    tot.core_calls = e->core_calls - core0;
    tot.core_kv_positions = e->core_kv_positions - kv0;
    tot.post_calls = e->post_calls - post0;
    tot.host_syncs = e->host_syncs - sync0;
    if (total) *total = tot;
  } catch (const std::exception& ex) {
    return fail(e, ex);
  }
  return LS_OK;
}
}  // namespace

int ls_generate(ls_engine* e, const int64_t* prompt, int n_prompt, int max_new, int mode,
                int64_t stop_token, int64_t* out_ids, int* n_out, ls_stats* stats) {
  if (!e || !n_out) return LS_EINVAL;
  const int32_t len = n_prompt;
  const uint64_t seed = e->sparams.seed;
  int32_t n = 0;
  const int rc = generate_batch(e, prompt, &len, 1, max_new, mode, {stop_rule(stop_token, nullptr, nullptr)},
                                &seed, out_ids, &n, nullptr, stats, stop_token < 0 ? -1 : stop_token);
  *n_out = n;
  return rc;
}

int ls_generate_stream(ls_engine* e, const int64_t* prompt, int n_prompt, int max_new, int mode,
                       int64_t stop_token, ls_commit_fn on_commit, void* user, int64_t* out_ids,
                       int* n_out, ls_stats* stats) {
  if (!e || !on_commit || !n_out) return LS_EINVAL;
  const int32_t len = n_prompt;
  const uint64_t seed = e->sparams.seed;
  int32_t n = 0;
  const int rc = generate_batch(e, prompt, &len, 1, max_new, mode, {stop_rule(stop_token, on_commit, user)},
                                &seed, out_ids, &n, nullptr, stats);
  *n_out = n;
  return rc;
}

int ls_generate_batch(ls_engine* e, const int64_t* prompts, const int32_t* prompt_lens, int n_requests,
                      int max_new_tokens, int mode, int64_t stop_token, const uint64_t* seeds,
                      int64_t* out_ids, int32_t* n_out, ls_stats* per_request, ls_stats* total) {
  if (!e || n_requests < 1) return LS_EINVAL;
  std::vector<StopRule> stops(n_requests, stop_rule(stop_token, nullptr, nullptr));
  return generate_batch(e, prompts, prompt_lens, n_requests, max_new_tokens, mode, stops, seeds, out_ids,
                        n_out, per_request, total);
}

int ls_generate_batch_sampling(ls_engine* e, const int64_t* prompts, const int32_t* prompt_lens,
                               int n_requests, int max_new_tokens, int mode, int64_t stop_token,
                               const uint64_t* seeds, const float* temperature, const int32_t* top_k,
                               const float* top_p, int64_t* out_ids, int32_t* n_out, ls_stats* per_request,
                               ls_stats* total) {
  if (!e || n_requests < 1 || !seeds || !temperature || !top_k || !top_p) return LS_EINVAL;
  std::vector<SampleParams> params(n_requests);
  for (int i = 0; i < n_requests; ++i) {
    if (!(temperature[i] >= 0.f && top_k[i] >= 0 && top_p[i] > 0.f && top_p[i] <= 1.f)) {
      e->last_error = "sampling needs temperature >= 0, top_k >= 0, 0 < top_p <= 1 (request " +
                      std::to_string(i) + ")";
      return LS_EINVAL;
    }
    params[i] = sample_params(temperature[i], top_k[i], top_p[i], seeds[i]);
  }
  std::vector<StopRule> stops(n_requests, stop_rule(stop_token, nullptr, nullptr));
  return generate_batch(e, prompts, prompt_lens, n_requests, max_new_tokens, mode, stops, seeds, out_ids,
                        n_out, per_request, total, -2, params.data());
}

namespace {
// The device loop's scheduler state compiled for the host, with capacities for
// every schedule (S <= 32, up to 256 live lanes).
using HostSched = DevSched<256, 4096, 32, 2048, 16384, 32768>;
// The same with a 4-slot id map, so that most lookups take the scan fallback.
using HostSchedNarrowMap = DevSched<256, 4096, 32, 2048, 16384, 32768, 4>;
constexpr int kSimRows = 16384;   // mapping rows of a simulated request
}  // namespace

extern "C++" {
namespace {

// Invariants of a scheduler's node, cursor and row tables: the ascending-id
// list holds exactly the nodes in use, every node is found by its id, the id
// map and unmapped count agree with the nodes (an unmapped node's slot may
// have emptied since), and the cursors of the nodes in use are distinct, in
// use, and on distinct rows that are not free.
template <class D>
void check_tables(const D& d, std::vector<int>& row_seen, std::vector<int>& cur_seen) {
  int n_used = 0;
  for (int i = 0; i < (int)(sizeof(d.nodes) / sizeof(d.nodes[0])); ++i) n_used += d.nodes[i].used;
  int n_list = 0, n_unmapped = 0, prev = -1;
  for (int i = d.node_head; i >= 0; i = d.nodes[i].next) {
    const auto& n = d.nodes[i];
    REQUIRE(n.used && n.prev == prev && (prev < 0 || d.nodes[prev].id < n.id), LS_EPIPELINE,
            "device scheduler: node list out of order");
    REQUIRE(d.node_of(n.id) == i, LS_EPIPELINE, "device scheduler: node lookup failed");
    const int h = n.id & (D::kIdSlots - 1);
    REQUIRE(n.mapped ? d.id_slot[h] == i : d.id_slot[h] != i, LS_EPIPELINE,
            "device scheduler: id map out of step");
    n_unmapped += !n.mapped;
    prev = i;
    ++n_list;
  }
  REQUIRE(n_list == n_used && d.node_tail == prev && n_unmapped == d.n_unmapped, LS_EPIPELINE,
          "device scheduler: node list incomplete");
  std::fill(row_seen.begin(), row_seen.end(), 0);
  std::fill(cur_seen.begin(), cur_seen.end(), 0);
  for (int k = 0; k < d.n_free_rows; ++k) row_seen[d.free_rows[k]] += 1;
  for (int i = d.node_head; i >= 0; i = d.nodes[i].next)
    for (int r = 0; r < 3; ++r)
      for (int t = 0; t < d.S; ++t) {
        const int c = d.nodes[i].cur[r][t];
        if (c < 0) continue;
        REQUIRE(d.cursors[c].used && cur_seen[c]++ == 0, LS_EPIPELINE, "device scheduler: cursor shared or freed");
        row_seen[d.cursors[c].row] += 1;
      }
  for (int v : row_seen)
    REQUIRE(v == 1, LS_EPIPELINE, "device scheduler: mapping row lost or shared");
}

// Start a simulated request: rows 0..kSimRows-1 free, unbounded KV slots, and
// root cursors for every role and depth, so that plan() forks and releases
// timelines as on the GPU.
template <class D>
void sim_start(D& d, int S, int K, int X, int max_rows, int max_new, long long stop_token, long long first,
               long long* out) {
  ds_start(d, S, K, X, max_rows, max_new, stop_token, first, out);
  d.has_pre = d.has_post = 1;
  d.n_free_rows = kSimRows;
  for (int r = 0; r < kSimRows; ++r) d.free_rows[r] = kSimRows - 1 - r;
  d.next_slot = 0;
  d.slot_limit = 0x7fffffff;
  for (int r = 0; r < 3; ++r)
    for (int t = 0; t < S; ++t) d.nodes[0].cur[r][t] = d.new_cursor(d.alloc_row(), 0, -1);
}

template <class D>
void sim_plan(D& d, std::vector<DsFill>& pre, std::vector<DsFill>& core, std::vector<DsFill>& post) {
  int n_pre = 0, n_post = 0;
  d.plan(pre.data(), n_pre, core.data(), post.data(), n_post);
}
}  // namespace
}  // extern "C++"

int ls_device_loop_simulate(int stages, int step_size, int second_step, int64_t first_token,
                            int max_new_tokens, int64_t stop_token, ls_decide_fn decide,
                            ls_cycle_fn on_cycle, ls_retain_fn on_retain, void* user,
                            int64_t* out_ids, int* n_out, ls_stats* stats) {
  if (!decide || !out_ids || !n_out || max_new_tokens < 1) return LS_EINVAL;
  try {
    const int S = stages, K = step_size, X = second_step;
    REQUIRE(S > 0 && S <= 32, LS_EINVAL, "stages S must be in 1..32");
    REQUIRE(K >= 1 && K < S && S % K == 0, LS_EINVAL, "step_size K must be a positive divisor of S with K < S");
    REQUIRE(X == 0 || (X > 1 && X < S / K), LS_EINVAL, "second_step X must satisfy 1 < X < S/K");
    const int depth = S / K;
    std::vector<long> b;
    if (X == 0) b.assign(depth, 1);
    else {
      b.assign(X, 1);
      for (int t = X; t < depth; ++t) b.push_back(b[t - 1] + b[t - X]);
    }
    int max_rows = 0;
    for (long v : b) max_rows += (int)v;
    REQUIRE(max_rows <= 256, LS_ECAPACITY, "schedule needs more than 256 lanes");
    // the scheduler, and a shadow with a 4-slot id map fed the same decisions:
    // apart from their id maps the two must stay identical
    std::unique_ptr<HostSched> d(new HostSched());
    std::unique_ptr<HostSchedNarrowMap> w(new HostSchedNarrowMap());
    std::vector<long long> out(max_new_tokens), out_w(max_new_tokens);
    sim_start(*d, S, K, X, max_rows, max_new_tokens, stop_token, first_token, out.data());
    sim_start(*w, S, K, X, max_rows, max_new_tokens, stop_token, first_token, out_w.data());
    std::vector<DsFill> pre(256), core(256 * 32), post(256);
    std::vector<int> row_seen(kSimRows), cur_seen(16384);
    auto check = [&]() {
      check_tables(*d, row_seen, cur_seen);
      check_tables(*w, row_seen, cur_seen);
      bool same = d->n_lanes == w->n_lanes && d->committed == w->committed && d->err == w->err &&
                  d->done == w->done && d->next_slot == w->next_slot && d->n_free_rows == w->n_free_rows;
      for (int i = 0; same && i < d->n_lanes; ++i)
        same = std::memcmp(&d->lanes[i], &w->lanes[i], sizeof(DsLane)) == 0;
      for (int i = 0; same && i < (int)(sizeof(d->nodes) / sizeof(d->nodes[0])); ++i) {
        const auto &a = d->nodes[i], &b = w->nodes[i];
        same = a.used == b.used &&
               (!a.used || (a.id == b.id && a.parent == b.parent && a.child_count == b.child_count &&
                            a.live == b.live && a.prev == b.prev && a.next == b.next &&
                            std::memcmp(a.cur, b.cur, sizeof(a.cur)) == 0));
      }
      REQUIRE(same, LS_EPIPELINE, "device scheduler: the narrow-map shadow diverged");
    };
    check();
    auto report_retain = [&]() {
      std::vector<int64_t> pairs;
      for (int i = 0; i < d->n_lanes; ++i) {
        pairs.push_back(d->lanes[i].branch);
        pairs.push_back(d->lanes[i].parent);
      }
      if (on_retain) on_retain(user, pairs.data(), (int32_t)d->n_lanes, d->last_accepted);
    };
    if (d->done) report_retain();
    std::vector<long long> dec;
    while (!d->done && !d->err) {
      const int n = d->gather();
      w->gather();
      sim_plan(*d, pre, core, post);
      sim_plan(*w, pre, core, post);
      std::vector<int64_t> rows;
      dec.assign(n, -1);
      for (int i = 0; i < n; ++i) {
        const DsLane& l = d->lanes[i];
        const int64_t r[7] = {l.stage, l.index, l.token, l.branch, l.parent, l.origin, l.state};
        rows.insert(rows.end(), r, r + 7);
        const int kind = d->kind_of[l.stage + K - 1];
        if (kind >= 0) dec[i] = decide(user, l.index, l.token, kind);
      }
      if (on_cycle) on_cycle(user, rows.data(), (int32_t)n);
      d->consume(dec.data(), 1, out.data());
      w->consume(dec.data(), 1, out_w.data());
      check();
      report_retain();
    }
    REQUIRE(d->err == kDsOk, LS_EPIPELINE, "device scheduler reported error " + std::to_string(d->err));
    ls_stats st{};
    st.pipeline_cycles = d->stats[0];
    st.pre_rows = d->stats[1];
    st.recurrent_rows = d->stats[2];
    st.post_rows = d->stats[3];
    st.verified_proposals = d->stats[4];
    st.first_rejections = d->stats[5];
    st.second_verifications = d->stats[6];
    st.second_acceptances = d->stats[7];
    st.second_rejections = d->stats[8];
    st.decode_tokens = std::max(d->committed - 1, 0);
    for (int i = 0; i < d->committed; ++i) out_ids[i] = out[i];
    *n_out = d->committed;
    if (stats) *stats = st;
  } catch (const std::exception& ex) {
    return fail(nullptr, ex);
  }
  return LS_OK;
}

int ls_pipeline_simulate(int stages, int step_size, int second_step, int64_t first_token,
                         int max_new_tokens, int64_t stop_token, ls_decide_fn decide,
                         ls_cycle_fn on_cycle, ls_retain_fn on_retain, void* user,
                         int64_t* out_ids, int* n_out, ls_stats* stats) {
  if (!decide || !out_ids || !n_out || max_new_tokens < 1) return LS_EINVAL;
  try {
    const int S = stages, K = step_size, X = second_step;
    REQUIRE(S > 0, LS_EINVAL, "stages S must be a positive integer");
    REQUIRE(K >= 1 && K < S && S % K == 0, LS_EINVAL, "step_size K must be a positive divisor of S with K < S");
    REQUIRE(X == 0 || (X > 1 && X < S / K), LS_EINVAL, "second_step X must satisfy 1 < X < S/K");
    SchedHooks hk;
    hk.S = S;
    hk.K = K;
    hk.X = X;
    hk.endpoint_kind[K - 1] = 0;
    if (X) hk.endpoint_kind[K * X - 1] = 1;
    hk.endpoint_kind[S - 1] = 2;
    const int depth = S / K;
    std::vector<long> b;
    if (X == 0) b.assign(depth, 1);
    else {
      b.assign(X, 1);
      for (int t = X; t < depth; ++t) b.push_back(b[t - 1] + b[t - X]);
    }
    for (long v : b) hk.max_rows += (int)v;
    Forward forward = [&](const std::vector<CycleLane>& cl, std::vector<Dec>& dec) {
      std::vector<int64_t> rows;
      for (auto& l : cl) {
        const int64_t r[7] = {l.stage, l.index, l.token, l.branch, l.parent, l.origin, l.state};
        rows.insert(rows.end(), r, r + 7);
      }
      if (on_cycle) on_cycle(user, rows.data(), (int32_t)cl.size());
      dec.assign(cl.size(), Dec{-1, 0, 0, 0, 0});
      for (size_t i = 0; i < cl.size(); ++i) {
        auto it = hk.endpoint_kind.find(cl[i].stage + K - 1);
        if (it != hk.endpoint_kind.end()) dec[i][0] = decide(user, cl[i].index, cl[i].token, it->second);
      }
    };
    hk.retain = [&](const std::vector<PLane>& lanes, int accepted) {
      std::vector<int64_t> pairs;
      for (auto& l : lanes) {
        pairs.push_back(l.branch);
        pairs.push_back(l.parent);
      }
      if (on_retain) on_retain(user, pairs.data(), (int32_t)lanes.size(), accepted);
    };
    hk.should_stop = [stop_token](const std::vector<long long>& ids) {
      return stop_token >= 0 && ids.back() == stop_token;
    };
    double t0 = -1.0;
    std::vector<std::unique_ptr<PipelineRun>> runs;
    runs.emplace_back(new PipelineRun(hk, 0, 0, first_token, max_new_tokens, &t0));
    drive(runs, forward);
    ls_stats st = runs[0]->st;
    const std::vector<long long>& ids = runs[0]->committed;
    st.decode_tokens = std::max<int64_t>((int64_t)ids.size() - 1, 0);
    for (size_t i = 0; i < ids.size(); ++i) out_ids[i] = ids[i];
    *n_out = (int)ids.size();
    if (stats) *stats = st;
  } catch (const std::exception& ex) {
    return fail(nullptr, ex);
  }
  return LS_OK;
}

int ls_role_kernel_count(ls_engine* e, int role, int n, int* count) {
  if (!e || !count || role < 0 || role > 2 || n < 1) return LS_EINVAL;
  try {
    REQUIRE(e->finalized, LS_EINVAL, "engine not finalized");
    // Count by capturing the chain into a throwaway graph.
    CK(cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal));
    try {
      enqueue_role(*e, role, n);
    } catch (...) {
      cudaGraph_t g = nullptr;
      cudaStreamEndCapture(e->stream, &g);
      if (g) cudaGraphDestroy(g);
      throw;
    }
    cudaGraph_t g = nullptr;
    CK(cudaStreamEndCapture(e->stream, &g));
    size_t nodes = 0;
    cudaGraphGetNodes(g, nullptr, &nodes);
    cudaGraphDestroy(g);
    *count = (int)nodes;
  } catch (const std::exception& ex) {
    return fail(e, ex);
  }
  return LS_OK;
}

int ls_time_role(ls_engine* e, int role, int n, int context_len, int iters, double* avg_ms) {
  if (!e || !avg_ms || role < 0 || role > 2 || n < 1 || iters < 1) return LS_EINVAL;
  try {
    Request& R = e->reqs.at(0);
    REQUIRE(R.prefill_len >= 0, LS_EINVAL, "ls_time_role needs a prefilled request");
    REQUIRE(n <= e->max_state, LS_ECAPACITY, "too many lanes");
    const int P = R.prefill_len + 1;
    REQUIRE(context_len >= 1 && context_len <= P, LS_EINVAL, "context_len must not exceed the prompt");
    // Synthetic lanes, as decode lanes at different depths: lane b gets a
    // fresh row forking the request's timeline of depth b mod S (core; pre
    // and post have one depth) at context_len - 1 and appends one token
    // there, so up to S lanes read distinct K/V. The fork runs once, in a
    // warm-up call; the timed calls only append, like decode calls. This
    // overwrites nothing of the request's timelines but consumes rows/slots
    // until the next ls_prefill, which resets the pools.
    const bool attn = role == kCore || (role == kPre && e->mc.n_pre_layers) ||
                      (role == kPost && e->mc.n_post_layers);
    int* m = stage_meta(*e);
    for (int b = 0; b < n; ++b) {
      Cursor c;
      if (attn) {
        const int depth = role == kPost ? e->S - 1 : role == kCore ? b % e->S : 0;
        Cursor* root = R.tl.get_or_create_cursor(role, depth, 0, -1);
        c.row = R.tl.alloc_row();
        c.seq_len = context_len - 1;
        c.pending_parent_row = root->row;
      }
      fill_lane(*e, R.tl, m, b, 1, context_len - 1, attn ? &c : nullptr, b, b);
      // post lanes read out as final verifications without a proposal
      if (role == kPost) set_final_readout(*e, m, b, R, 1, b);
    }
    run_role(*e, role, n, m, true);  // forks the rows
    int* m2 = stage_meta(*e);
    std::copy(m, m + kMetaFields * e->cap, m2);
    for (int b = 0; b < n; ++b) {
      put(*e, m2, kMetaForkRow, b, -1);
      put(*e, m2, kMetaForkLen, b, 0);
    }
    run_role(*e, role, n, m2, true);  // warm-up of the append-only call (captures its graph)
    CK(cudaEventRecord(e->ev0, e->stream));
    for (int i = 0; i < iters; ++i) run_role(*e, role, n, m2, true);
    CK(cudaEventRecord(e->ev1, e->stream));
    CK(cudaEventSynchronize(e->ev1));
    e->staging_next = 0;
    check_device(*e);
    float ms = 0.f;
    CK(cudaEventElapsedTime(&ms, e->ev0, e->ev1));
    *avg_ms = ms / iters;
  } catch (const std::exception& ex) {
    return fail(e, ex);
  }
  return LS_OK;
}

int ls_time_gemm(ls_engine* e, int which, int n, int iters, double* avg_ms) {
  if (!e || !avg_ms || which < 0 || which > 4 || n < 1 || iters < 1) return LS_EINVAL;
  try {
    REQUIRE(e->finalized, LS_EINVAL, "engine not finalized");
    REQUIRE(n <= e->cap, LS_ECAPACITY, "too many lanes");
    LayerW& w = e->core.layers[0];
    const Gemm* g[] = {&w.g_qkv, &w.g_o, &w.g_gu, &w.g_down, &e->g_lm};
    XBuf* x[] = {&e->x_h, &e->x_attn, &e->x_h, &e->x_act, &e->x_h};
    float* out = which == 4 ? e->logits : e->part;
    gemm_store(*e, *g[which], *x[which], out, n);
    CK(cudaEventRecord(e->ev0, e->stream));
    for (int i = 0; i < iters; ++i) gemm_store(*e, *g[which], *x[which], out, n);
    CK(cudaEventRecord(e->ev1, e->stream));
    CK(cudaEventSynchronize(e->ev1));
    check_device(*e);
    float ms = 0.f;
    CK(cudaEventElapsedTime(&ms, e->ev0, e->ev1));
    *avg_ms = ms / iters;
  } catch (const std::exception& ex) {
    return fail(e, ex);
  }
  return LS_OK;
}

int ls_debug_gemm(ls_engine* e, int which, int n, const float* x_host, float* out_host) {
  if (!e || !x_host || !out_host || which < 0 || which > 5 || n < 1) return LS_EINVAL;
  try {
    REQUIRE(e->finalized, LS_EINVAL, "engine not finalized");
    REQUIRE(n <= e->cap, LS_ECAPACITY, "too many lanes");
    REQUIRE(which != 5 || e->mc.family == LS_FAMILY_RAVEN, LS_EINVAL, "no adapter in this model");
    LayerW& w = e->core.layers[0];
    const Gemm* g[] = {&w.g_qkv, &w.g_o, &w.g_gu, &w.g_down, &e->g_lm, &e->g_adapter};
    XBuf* x[] = {&e->x_h, &e->x_attn, &e->x_h, &e->x_act, &e->x_h, &e->x_cat};
    const Gemm& gm = *g[which];
    XBuf& xb = *x[which];
    std::vector<bf16> xs((size_t)2 * n * gm.K);
    for (int b = 0; b < n; ++b)
      for (int k = 0; k < gm.K; ++k) {
        const float v = x_host[(size_t)b * gm.K + k];
        const bf16 hi = __float2bfloat16_rn(v);
        xs[(size_t)(2 * b) * gm.K + k] = hi;
        xs[(size_t)(2 * b + 1) * gm.K + k] = __float2bfloat16_rn(v - __bfloat162float(hi));
      }
    CK(cudaMemcpyAsync(xb.ptr, xs.data(), sizeof(bf16) * xs.size(), cudaMemcpyHostToDevice, e->stream));
    CK(cudaStreamSynchronize(e->stream));
    float* out = which == 4 ? e->logits : e->part;
    gemm_store(*e, gm, xb, out, n);
    CK(cudaMemcpyAsync(out_host, out, sizeof(float) * (size_t)n * gm.Mw, cudaMemcpyDeviceToHost,
                       e->stream));
    CK(cudaStreamSynchronize(e->stream));
    check_device(*e);
  } catch (const std::exception& ex) {
    return fail(e, ex);
  }
  return LS_OK;
}

int ls_gemm_splits(ls_engine* e, int which, int* splits, int* rows, int* k) {
  if (!e || !e->finalized || which < 0 || which > 5) return LS_EINVAL;
  LayerW& w = e->core.layers[0];
  const Gemm* g[] = {&w.g_qkv, &w.g_o, &w.g_gu, &w.g_down, &e->g_lm, &e->g_adapter};
  if (splits) *splits = g[which]->splits;
  if (rows) *rows = g[which]->Mw;
  if (k) *k = g[which]->K;
  return LS_OK;
}

int ls_time_core_gemms(ls_engine* e, int n, int iters, double* avg_launch_ms, double* bytes_per_launch) {
  if (!e || !avg_launch_ms || !bytes_per_launch || n < 1 || iters < 1) return LS_EINVAL;
  try {
    REQUIRE(e->finalized, LS_EINVAL, "engine not finalized");
    REQUIRE(n <= e->cap, LS_ECAPACITY, "too many lanes");
    double bytes = 0.0;
    int launches = 0;
    auto sweep = [&](bool count) {
      for (LayerW& w : e->core.layers) {
        const Gemm* g[] = {&w.g_qkv, &w.g_o, &w.g_gu, &w.g_down};
        XBuf* x[] = {&e->x_h, &e->x_attn, &e->x_h, &e->x_act};
        for (int i = 0; i < 4; ++i) {
          if (i == 2) {
            GemmEpi eg{};
            eg.x_act = e->x_act.ptr;
            eg.I = e->I;
            gemm(*e, *g[i], *x[i], eg, kEpiSwiGLU, n);
          } else {
            gemm_split_store(*e, *g[i], *x[i], n);   // the decode path's form (split planes)
          }
          if (count) {
            // weights + (hi, lo) activation rows read + outputs written (the
            // algorithmic output; split planes add splits x that, not counted)
            const double out_b = i == 2 ? 2.0 * 2 * n * (g[i]->Mw / 2) : 4.0 * n * g[i]->Mw;
            bytes += 2.0 * g[i]->Mw * g[i]->K + 2.0 * 2 * n * g[i]->K + out_b;
            launches++;
          }
        }
      }
    };
    sweep(false);
    CK(cudaEventRecord(e->ev0, e->stream));
    for (int it = 0; it < iters; ++it) sweep(it == 0);
    CK(cudaEventRecord(e->ev1, e->stream));
    CK(cudaEventSynchronize(e->ev1));
    check_device(*e);
    float ms = 0.f;
    CK(cudaEventElapsedTime(&ms, e->ev0, e->ev1));
    *avg_launch_ms = ms / (iters * launches);
    *bytes_per_launch = bytes / launches;
  } catch (const std::exception& ex) {
    return fail(e, ex);
  }
  return LS_OK;
}

int ls_debug_kv(ls_engine* e, void** k, void** v, int* slots, int* layers) {
  if (!e || !e->finalized) return LS_EINVAL;
  if (k) *k = e->kpool;
  if (v) *v = e->vpool;
  if (slots) *slots = e->n_slots;
  if (layers) *layers = e->n_attn_layers;
  return LS_OK;
}

int ls_destroy(ls_engine* e) {
  if (!e) return LS_EINVAL;
  if (e->stream) cudaStreamSynchronize(e->stream);
  delete e;
  return LS_OK;
}

}  // extern "C"
