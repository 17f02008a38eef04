// The LoopSpec scheduler of one request as fixed-size state that a
// single GPU thread can run between the role calls of a cycle, so that whole
// cycles run back to back without a host round trip.
//
// It restates, with arrays instead of maps and heaps:
//   continue_pipelined (sglang_recurrent/loopspec/pipeline.py:254-423) with
//     greedy resolve (loopspec/decisions.py:136-184) or the sampled decision
//     rows' resolve (loopspec/sampling/policy.py:285-308), the executor's
//     state-slot pool and counters (loopspec/executor.py:76-107, 239-290);
//   the branch timeline bookkeeping (loopspec/branching/manager.py:45-482):
//     cursors per (branch, role, depth), forks that share a parent's prefix,
//     ownership transfer to a single surviving child and recursive release.
// The engine's host scheduler (engine.cu, PipelineRun and Timelines) runs the
// same steps; the host-compiled instantiation of this code is checked against
// traces of the reference scheduler (ls_device_loop_simulate).
//
// KV slots are handed out in increasing order and not recycled before the
// request ends (the request's pool is sized for that); mapping rows are
// recycled when a cursor is released. Neither choice changes any lane's
// numbers: a timeline reads its positions through its mapping row.
//
// Every function is __host__ __device__; on the GPU one thread runs it on a
// copy of the state held in shared memory.
#pragma once

#include <stddef.h>
#include <stdint.h>

#include "common.cuh"

namespace ls {

#define LS_HD __host__ __device__ __forceinline__

enum DsError : int {
  kDsOk = 0,
  kDsNoStateSlot = 1,      // pipeline needs more recurrent state slots than configured
  kDsNoRow = 2,            // mapping rows exhausted
  kDsNoSlot = 3,           // KV slots exhausted
  kDsParent = 4,           // branch with an unavailable parent / missing parent timeline
  kDsFinal = 5,            // several lanes reached the final stage in one cycle
  kDsOrder = 6,            // commit out of order
  kDsTree = 7,             // speculative tree exceeded the row limit / capacity
  kDsDrained = 8,          // pipeline drained before generation completed
  kDsCapacity = 9,         // a fixed table of this state is full
};

constexpr int pow2_at_least(int n) {
  int p = 1;
  while (p < n) p *= 2;
  return p;
}

struct DsLane {
  int stage, index, token, state, branch, parent, origin, first, second;
};

template <int MAXD>
struct DsNode {
  int id, parent, child_count, live, used;
  int prev, next;     // neighbours in the list of nodes in use by ascending id (-1: none)
  int mapped;         // 1 if the id map's slot of `id` holds this node
  int cur[3][MAXD];   // cursor index per (role, depth), -1 if none
};

struct DsCursor {
  int row, seq_len, pending_parent_row, used;
};

// One lane of a role call, as the host's fill_lane() describes it.
struct DsFill {
  int token, pos, row, slot, fork_row, fork_len, state_in, state_out;
  int kind, first, second;   // post rows
};

template <int MAXL, int MAXB, int MAXD, int MAXN, int MAXC, int MAXR, int IDS = pow2_at_least(4 * MAXN)>
struct alignas(16) DevSched {
  // schedule and request
  int S, K, X, max_rows, max_new, q1, q2, final_stage;
  int kind_of[MAXD];          // end stage -> 0 q1, 1 q2, 2 final, -1 none
  int has_pre, has_post;      // pre / post roles with attention layers
  long long stop_token;
  int prefill_len, state_base;
  // pipeline
  int n_lanes;
  DsLane lanes[MAXL];
  // ancestry: branch -> parent (-1 for the root), an open-addressing table
  // keyed by branch id (linear probing, -1 = empty; rebuilt whole by
  // prune_ancestry, so entries are never deleted one by one)
  static constexpr int kParSlots = pow2_at_least(2 * MAXB);
  int n_par;
  int par_key[kParSlots], par_val[kParSlots];
  int next_branch;
  unsigned char state_used[MAXL];
  int committed, done, err;
  int draw_cycle;             // random-stream cycle counter of the request's readouts
  unsigned long long seed;    // the request's sampling seed (Philox key of its draws)
  long long kv_positions;     // sum over core lanes of the timeline length attended
  long long last_token;
  int last_accepted;          // accepted stage of the last retention (-1: none)
  long long stats[9];   // pipeline_cycles, pre_rows, recurrent_rows, post_rows, verified_proposals,
                        // first_rejections, second_verifications, second_acceptances, second_rejections
  // timelines
  static constexpr int kNodeWords = (MAXN + 63) / 64, kCurWords = (MAXC + 63) / 64;
  // branch id -> node index, direct-mapped on id mod kIdSlots (-1 = empty).
  // Live ids are a narrow window of a counter, so two nodes in use rarely
  // share a slot; one that finds its slot taken is counted in n_unmapped and
  // found by a scan.
  static constexpr int kIdSlots = IDS;
  static_assert((IDS & (IDS - 1)) == 0, "the id map's size is a power of two");
  DsNode<MAXD> nodes[MAXN];
  DsCursor cursors[MAXC];
  int id_slot[kIdSlots];
  int n_unmapped;
  int node_head, node_tail;                   // ends of the ascending-id list
  unsigned long long node_bits[kNodeWords];   // bit i: nodes[i] in use
  unsigned long long cur_bits[kCurWords];     // bit i: cursors[i] in use
  int n_free_rows;
  int free_rows[MAXR];
  int next_slot, slot_limit;

  // ------------------------------------------------------------ helpers
  LS_HD void fail(int code) {
    if (!err) err = code;
  }

  // Lowest set (or, inverted, clear) bit of a word array; -1 if none. A
  // scan of the bits visits only the entries in use, in increasing index.
  static LS_HD int ctz64(unsigned long long x) {
#ifdef __CUDA_ARCH__
    return __ffsll((long long)x) - 1;
#else
    return __builtin_ctzll(x);
#endif
  }
  template <int W>
  static LS_HD int first_clear(const unsigned long long (&bits)[W], int limit) {
    for (int w = 0; w < W; ++w)
      if (~bits[w]) {
        const int i = w * 64 + ctz64(~bits[w]);
        return i < limit ? i : -1;
      }
    return -1;
  }
  // the node of branch `id`, or -1: one id-map probe, a scan of the nodes in
  // use only while some node is unmapped
  LS_HD int node_of(int id) const {
    if (id < 0) return -1;
    const int m = id_slot[id & (kIdSlots - 1)];
    if (m >= 0 && nodes[m].id == id) return m;   // a slot only ever holds a node in use
    if (n_unmapped == 0) return -1;
    for (int w = 0; w < kNodeWords; ++w)
      for (unsigned long long m = node_bits[w]; m; m &= m - 1) {
        const int i = w * 64 + ctz64(m);
        if (nodes[i].id == id) return i;
      }
    return -1;
  }

  // slot of branch b, or of the empty slot where it would go
  LS_HD int par_slot(int b) const {
    int h = b & (kParSlots - 1);
    for (int k = 0; k < kParSlots; ++k, h = (h + 1) & (kParSlots - 1))
      if (par_key[h] == b || par_key[h] < 0) return h;
    return -1;   // full (cannot happen: at most MAXB of kParSlots >= 2 MAXB slots are used)
  }

  LS_HD int parent_of(int b) const {
    const int h = b < 0 ? -1 : par_slot(b);
    return h >= 0 && par_key[h] == b ? par_val[h] : -2;   // -2: unknown branch
  }

  LS_HD void set_parent(int b, int p) {
    const int h = par_slot(b);
    if (h >= 0 && par_key[h] == b) {
      par_val[h] = p;
      return;
    }
    if (h < 0 || n_par >= MAXB) {
      fail(kDsCapacity);
      return;
    }
    par_key[h] = b;
    par_val[h] = p;
    ++n_par;
  }

  LS_HD void clear_parents() {
    for (int i = 0; i < kParSlots; ++i) par_key[i] = -1;
    n_par = 0;
  }

  LS_HD int alloc_row() {
    if (n_free_rows <= 0) {
      fail(kDsNoRow);
      return 0;
    }
    return free_rows[--n_free_rows];
  }

  LS_HD void free_row(int r) {
    if (n_free_rows < MAXR) free_rows[n_free_rows++] = r;
  }

  LS_HD int alloc_slot() {
    if (next_slot >= slot_limit) {
      fail(kDsNoSlot);
      return 0;
    }
    return next_slot++;
  }

  LS_HD int new_cursor(int row, int seq_len, int pending) {
    const int i = first_clear(cur_bits, MAXC);   // the lowest free entry
    if (i < 0) {
      fail(kDsCapacity);
      return 0;
    }
    cur_bits[i / 64] |= 1ull << (i % 64);
    cursors[i].used = 1;
    cursors[i].row = row;
    cursors[i].seq_len = seq_len;
    cursors[i].pending_parent_row = pending;
    return i;
  }

  LS_HD int new_node(int id, int parent) {
    const int i = first_clear(node_bits, MAXN);   // the lowest free entry
    if (i < 0) {
      fail(kDsCapacity);
      return 0;
    }
    node_bits[i / 64] |= 1ull << (i % 64);
    DsNode<MAXD>& n = nodes[i];
    n.used = 1;
    n.id = id;
    n.parent = parent;
    n.child_count = 0;
    n.live = 1;
    for (int r = 0; r < 3; ++r)
      for (int d = 0; d < MAXD; ++d) n.cur[r][d] = -1;
    int& slot = id_slot[id & (kIdSlots - 1)];
    n.mapped = slot < 0;
    if (n.mapped) slot = i;
    else ++n_unmapped;
    // ids come from a counter, so a new node almost always goes at the tail
    int t = node_tail;
    while (t >= 0 && nodes[t].id > id) t = nodes[t].prev;
    n.prev = t;
    n.next = t >= 0 ? nodes[t].next : node_head;
    if (n.next >= 0) nodes[n.next].prev = i;
    else node_tail = i;
    if (t >= 0) nodes[t].next = i;
    else node_head = i;
    return i;   // (depths >= S stay -1: loops below stop at S)
  }

  LS_HD void free_node(int i) {
    DsNode<MAXD>& n = nodes[i];
    n.used = 0;
    node_bits[i / 64] &= ~(1ull << (i % 64));
    if (n.mapped) id_slot[n.id & (kIdSlots - 1)] = -1;
    else --n_unmapped;
    if (n.prev >= 0) nodes[n.prev].next = n.next;
    else node_head = n.next;
    if (n.next >= 0) nodes[n.next].prev = n.prev;
    else node_tail = n.prev;
  }

  // an empty node table (before the root is created)
  LS_HD void clear_nodes() {
    for (int w = 0; w < kNodeWords; ++w) node_bits[w] = 0;
    for (int h = 0; h < kIdSlots; ++h) id_slot[h] = -1;
    n_unmapped = 0;
    node_head = node_tail = -1;
  }

  // -------------------------------------- timelines (manager.py:207-482)
  LS_HD int get_or_create_branch(int id, int parent_id) {
    int n = node_of(id);
    if (n >= 0) return n;
    const int p = node_of(parent_id);
    if (p < 0) {
      fail(kDsParent);
      return 0;
    }
    n = new_node(id, parent_id);
    nodes[p].child_count += 1;
    return n;
  }

  LS_HD int get_or_create_cursor(int role, int depth, int branch, int parent) {
    return cursor_of_node(get_or_create_branch(branch, parent), role, depth);
  }

  // the cursor of node n's timeline at (role, depth), forked from its parent's
  LS_HD int cursor_of_node(int n, int role, int depth) {
    if (nodes[n].cur[role][depth] >= 0) return nodes[n].cur[role][depth];
    const int p = nodes[n].parent < 0 ? -1 : node_of(nodes[n].parent);
    if (p < 0 || nodes[p].cur[role][depth] < 0) {
      fail(kDsParent);
      return 0;
    }
    const DsCursor& pc = cursors[nodes[p].cur[role][depth]];
    const int c = new_cursor(alloc_row(), pc.seq_len, pc.row);
    nodes[n].cur[role][depth] = c;
    return c;
  }

  LS_HD void release_cursor(int c) {
    free_row(cursors[c].row);
    cursors[c].used = 0;
    cur_bits[c / 64] &= ~(1ull << (c % 64));
  }

  LS_HD void release_unused(int n) {
    while (n >= 0 && !nodes[n].live && nodes[n].child_count == 0) {
      for (int r = 0; r < 3; ++r)
        for (int d = 0; d < S; ++d)
          if (nodes[n].cur[r][d] >= 0) release_cursor(nodes[n].cur[r][d]);
      const int pid = nodes[n].parent;
      free_node(n);
      if (pid < 0) break;
      const int p = node_of(pid);
      if (p < 0) break;
      nodes[p].child_count -= 1;
      n = p;
    }
  }

  LS_HD void detach_from_unused_parent(int n) {
    const int pid = nodes[n].parent;
    if (pid < 0) return;
    const int p = node_of(pid);
    if (p < 0 || nodes[p].live || nodes[p].child_count != 1) return;
    for (int r = 0; r < 3; ++r)
      for (int d = 0; d < S; ++d) {
        if (nodes[p].cur[r][d] < 0) continue;
        if (nodes[n].cur[r][d] < 0) {   // the child adopts the parent's timeline
          nodes[n].cur[r][d] = nodes[p].cur[r][d];
          nodes[p].cur[r][d] = -1;
        }
      }
    nodes[n].parent = -1;
    nodes[p].child_count -= 1;
    release_unused(p);
  }

  // keep the timelines of these (branch, parent) lanes, release the rest
  LS_HD void retain(const DsLane* keep, int nk) {
    // branches are created in (branch, parent) order
    int order[MAXL];
    for (int i = 0; i < nk; ++i) order[i] = i;
    for (int i = 1; i < nk; ++i)
      for (int j = i; j > 0; --j) {
        const DsLane &a = keep[order[j - 1]], &b = keep[order[j]];
        if (a.branch > b.branch || (a.branch == b.branch && a.parent > b.parent)) {
          const int t = order[j - 1];
          order[j - 1] = order[j];
          order[j] = t;
        } else {
          break;
        }
      }
    for (int i = 0; i < nk; ++i) {
      const DsLane& l = keep[order[i]];
      if (l.branch && node_of(l.branch) < 0) get_or_create_branch(l.branch, l.parent);
    }
    // unused live nodes, released from the highest id down
    unsigned long long kept[kNodeWords];
    for (int w = 0; w < kNodeWords; ++w) kept[w] = 0;
    for (int k = 0; k < nk; ++k) {
      const int n = node_of(keep[k].branch);
      if (n >= 0) kept[n / 64] |= 1ull << (n % 64);
    }
    int ids[MAXN];
    int nu = 0;
    for (int i = node_tail; i >= 0; i = nodes[i].prev)
      if (nodes[i].live && !(kept[i / 64] >> (i % 64) & 1)) ids[nu++] = i;
    for (int k = 0; k < nu; ++k) {
      const int n = ids[k];
      if (!nodes[n].used) continue;
      nodes[n].live = 0;
      release_unused(n);
    }
    // single surviving children adopt their dead parents' timelines (ascending id)
    int na = 0;
    for (int i = node_head; i >= 0; i = nodes[i].next) ids[na++] = i;
    for (int k = 0; k < na; ++k)   // no node is created here, so a freed index stays free
      if (nodes[ids[k]].used) detach_from_unused_parent(ids[k]);
  }

  // ------------------------------------ pipeline (pipeline.py:254-423)
  LS_HD int acquire_state() {
    for (int s = 0; s < max_rows; ++s)
      if (!state_used[s]) {
        state_used[s] = 1;
        return s;
      }
    fail(kDsNoStateSlot);
    return 0;
  }

  LS_HD bool descends_from(int b, int anc) const {
    while (b != -1 && b != anc) {
      const int p = parent_of(b);
      b = p == -2 ? -1 : p;
    }
    return b == anc;
  }

  // Give every lane a state slot (executor.forward); returns the lane count.
  LS_HD int gather() {
    for (int i = 0; i < n_lanes; ++i)
      if (lanes[i].state < 0) lanes[i].state = acquire_state();
    return n_lanes;
  }

  // One cycle's decisions, `stride` values per lane: greedy (stride 1) the
  // argmax token of the lane's readout; sampling (stride 5) the row (token,
  // proposed, accepted_code, q1_rejected, q2_rejected) of policy.py:197-283.
  // Lanes without a readout are ignored. Appends a committed token to `out`
  // (indexed by the committed count) when the final lane commits.
  LS_HD void consume(const long long* dec, int stride, long long* out) {
    stats[0] += 1;
    stats[2] += (long long)n_lanes * K;
    for (int i = 0; i < n_lanes; ++i) {
      stats[1] += lanes[i].stage == 0;
      stats[3] += kind_of[lanes[i].stage + K - 1] >= 0;
    }
    DsLane following[MAXL];
    int nf = 0;
    DsLane children[MAXL];
    int nc = 0;
    int final_idx = -1;
    long long final_pred = 0;
    int accepted_stage = -1;
    for (int i = 0; i < n_lanes; ++i) {
      DsLane l = lanes[i];
      const int end_stage = l.stage + K - 1;
      const int kind = kind_of[end_stage];
      const long long* d = dec + (long)i * stride;
      const long long pred = d[0];
      bool proposed = false, fr = false, sr = false;
      int acc = -1;
      if (stride >= 5) {   // sampling resolve (policy.py:285-308)
        proposed = d[1] != 0;
        acc = d[2] == 1 ? q1 : d[2] == 2 ? q2 : -1;
        fr = d[3] != 0;
        sr = d[4] != 0;
      } else {             // greedy resolve (decisions.py:136-184)
        proposed = kind == 0 || (kind == 1 && (l.first < 0 || pred != l.first));
        if (kind == 2 && l.first >= 0) {
          fr = pred != l.first;
          if (!fr) acc = q1;
          else if (l.second >= 0) {
            sr = pred != l.second;
            if (!sr) acc = q2;
          }
        }
      }
      if (end_stage == final_stage) {
        if (final_idx >= 0) fail(kDsFinal);
        final_idx = i;
        final_pred = pred;
        accepted_stage = acc;
        const bool sv = fr && l.second >= 0;
        stats[4] += 1;
        stats[5] += fr;
        stats[6] += sv;
        stats[7] += sv && acc == q2;
        stats[8] += sv && sr;
        continue;
      }
      l.stage = end_stage + 1;
      if ((end_stage == q1 || end_stage == q2) && kind >= 0 && proposed) {
        if (end_stage == q1) l.first = (int)pred;
        else l.second = (int)pred;
        if (l.index + 1 < max_new) {
          if (nc >= MAXL) {
            fail(kDsTree);
            return;
          }
          DsLane c{0, l.index + 1, (int)pred, -1, next_branch, l.branch, end_stage, -1, -1};
          children[nc++] = c;
          set_parent(next_branch, l.branch);
          next_branch++;
        }
      }
      if (nf >= MAXL) {
        fail(kDsTree);
        return;
      }
      following[nf++] = l;
    }
    for (int i = 0; i < nc; ++i) {
      if (nf >= MAXL) {
        fail(kDsTree);
        return;
      }
      following[nf++] = children[i];
    }
    if (final_idx >= 0) {
      const DsLane fl = lanes[final_idx];
      if (fl.index != committed) fail(kDsOrder);
      out[committed++] = final_pred;
      last_token = final_pred;
      if ((stop_token >= 0 && final_pred == stop_token) || committed >= max_new) {
        // the request ends: every branch is released
        n_lanes = 0;
        for (int s = 0; s < MAXL; ++s) state_used[s] = 0;
        last_accepted = -1;
        retain(lanes, 0);
        done = 1;
        return;
      }
      accepted_stage = fl.first >= 0 ? accepted_stage : -1;
      if (fl.index + 1 < max_new) {
        int sel = -1;
        for (int j = 0; j < nf; ++j) {
          const DsLane& c = following[j];
          if (c.parent == fl.branch && c.token == final_pred && c.origin == accepted_stage &&
              accepted_stage >= 0) {
            sel = j;
            break;
          }
        }
        int keep;
        if (sel < 0) {
          if (nf >= MAXL) {
            fail(kDsTree);
            return;
          }
          DsLane c{0, fl.index + 1, (int)final_pred, -1, next_branch, fl.branch, final_stage, -1, -1};
          set_parent(next_branch, fl.branch);
          next_branch++;
          following[nf++] = c;
          keep = c.branch;
        } else {
          keep = following[sel].branch;
        }
        int nk = 0;
        for (int j = 0; j < nf; ++j)
          if (descends_from(following[j].branch, keep)) following[nk++] = following[j];
        nf = nk;
        prune_ancestry(following, nf, keep);
      } else {
        nf = 0;
        accepted_stage = -1;
      }
    }
    if (nf > max_rows) fail(kDsTree);
    n_lanes = nf;
    for (int i = 0; i < nf; ++i) lanes[i] = following[i];
    // state-slot pool retention: free the slots of lanes that are gone
    unsigned char keep_s[MAXL];
    for (int s = 0; s < MAXL; ++s) keep_s[s] = 0;
    for (int i = 0; i < nf; ++i)
      if (lanes[i].state >= 0) keep_s[lanes[i].state] = 1;
    for (int s = 0; s < MAXL; ++s)
      if (!keep_s[s]) state_used[s] = 0;
    last_accepted = accepted_stage;
    retain(lanes, nf);
    if (nf == 0 && committed < max_new) fail(kDsDrained);
    if (committed >= max_new) done = 1;
  }

  // the live ancestry: the root and every ancestor of a lane up to it
  LS_HD void prune_ancestry(const DsLane* ls, int n, int root) {
    int live[MAXB];
    int nl = 0;
    live[nl++] = root;
    for (int i = 0; i < n; ++i) {
      int b = ls[i].branch;
      while (b != root) {
        const int p = parent_of(b);
        if (b == -1 || p == -2) {
          fail(kDsTree);
          return;
        }
        bool seen = false;
        for (int k = 0; k < nl && !seen; ++k) seen = live[k] == b;
        if (!seen) {
          if (nl >= MAXB) {
            fail(kDsCapacity);
            return;
          }
          live[nl++] = b;
        }
        b = p;
      }
    }
    int nb[MAXB], np[MAXB];
    for (int k = 0; k < nl; ++k) {
      nb[k] = live[k];
      np[k] = live[k] == root ? -1 : parent_of(live[k]);
    }
    clear_parents();
    for (int k = 0; k < nl; ++k) set_parent(nb[k], np[k]);
  }

  // ----------------------------------------- one cycle's role metadata
  // Fill the lanes of the cycle's role calls as the host's cycle() does:
  // pre for stage-0 lanes, K core iterations for all lanes, post for readout
  // lanes; cursors advance after each call. Returns counts through n_*.
  LS_HD void plan(DsFill* pre, int& n_pre, DsFill* core /*[K][MAXL]*/, DsFill* post, int& n_post) {
    n_pre = 0;
    n_post = 0;
    int cur[MAXL];
    // each lane's branch node, found (or created) once for the cycle's calls;
    // nodes are only created during planning, so the indices stay valid
    int node[MAXL];
    for (int i = 0; i < n_lanes; ++i) node[i] = get_or_create_branch(lanes[i].branch, lanes[i].parent);
    for (int i = 0; i < n_lanes; ++i) {
      const DsLane& l = lanes[i];
      if (l.stage != 0) continue;
      DsFill& f = pre[n_pre];
      cur[n_pre] = has_pre ? cursor_of_node(node[i], 0, 0) : -1;
      fill(f, l, cur[n_pre], -1, state_base + l.state);
      ++n_pre;
    }
    for (int j = 0; j < n_pre; ++j)
      if (cur[j] >= 0) advance(cur[j]);
    for (int off = 0; off < K; ++off) {
      for (int i = 0; i < n_lanes; ++i) {
        const DsLane& l = lanes[i];
        cur[i] = cursor_of_node(node[i], 1, l.stage + off);
        fill(core[off * MAXL + i], l, cur[i], state_base + l.state, state_base + l.state);
        kv_positions += prefill_len + l.index + 1;
      }
      for (int i = 0; i < n_lanes; ++i) advance(cur[i]);
    }
    for (int i = 0; i < n_lanes; ++i) {
      const DsLane& l = lanes[i];
      const int end = l.stage + K - 1;
      if (kind_of[end] < 0) continue;
      DsFill& f = post[n_post];
      cur[n_post] = has_post ? cursor_of_node(node[i], 2, end) : -1;
      fill(f, l, cur[n_post], state_base + l.state, -1);
      f.kind = kind_of[end];
      f.first = l.first;
      f.second = l.second;
      ++n_post;
    }
    for (int j = 0; j < n_post; ++j)
      if (cur[j] >= 0) advance(cur[j]);
  }

  LS_HD void fill(DsFill& f, const DsLane& l, int c, int state_in, int state_out) {
    f.token = l.token;
    f.pos = prefill_len + l.index;
    f.state_in = state_in;
    f.state_out = state_out;
    f.kind = -1;
    f.first = -1;
    f.second = -1;
    if (c < 0) {
      f.row = f.slot = f.fork_row = -1;
      f.fork_len = 0;
      return;
    }
    const DsCursor& cu = cursors[c];
    f.row = cu.row;
    f.slot = alloc_slot();
    f.fork_row = cu.pending_parent_row;
    f.fork_len = cu.pending_parent_row >= 0 ? cu.seq_len : 0;
  }

  LS_HD void advance(int c) {
    cursors[c].pending_parent_row = -1;
    cursors[c].seq_len += 1;
  }
};

#undef LS_HD

}  // namespace ls

namespace ls {

// Start one request's pipeline after its first token (executor.py:400-434):
// the schedule, a live root branch 0 and one lane at stage 0 feeding `first`.
// The root's timelines (cursors) are attached by the caller.
template <class D>
inline void ds_start(D& d, int S, int K, int X, int max_rows, int max_new, long long stop_token,
                     long long first, long long* out) {
  d.S = S;
  d.K = K;
  d.X = X;
  d.max_rows = max_rows;
  d.max_new = max_new;
  d.q1 = K - 1;
  d.q2 = X ? K * X - 1 : -1;
  d.final_stage = S - 1;
  for (int i = 0; i < (int)(sizeof(d.kind_of) / sizeof(int)); ++i) d.kind_of[i] = -1;
  d.kind_of[K - 1] = 0;
  if (X) d.kind_of[K * X - 1] = 1;
  d.kind_of[S - 1] = 2;
  d.stop_token = stop_token;
  d.next_branch = 1;
  d.clear_parents();
  d.set_parent(0, -1);
  d.clear_nodes();
  d.new_node(0, -1);
  d.committed = 1;
  out[0] = first;
  d.last_token = first;
  d.last_accepted = -1;
  if ((stop_token >= 0 && first == stop_token) || max_new <= 1) {
    d.done = 1;
    return;
  }
  d.n_lanes = 1;
  d.lanes[0] = DsLane{0, 1, (int)first, -1, 0, -1, -1, -1, -1};
}

}  // namespace ls

namespace ls {

// ------------------------------------------------ device-resident decode loop
// The scheduler of one request for the device loop: up to 16 live
// lanes, S <= 8, 64 branch nodes, 128 cursors, 512 mapping rows.
using LoopSched = DevSched<16, 64, 8, 64, 128, 512>;
constexpr int kLoopMaxLanes = 16;
constexpr int kLoopMaxK = 8;
constexpr int kLoopThreads = 256;

// Lane metadata of one role call at a fixed width: `n` active lanes, the rest
// inactive (position -1), which every per-lane kernel skips. Fields 0..10 are
// DsFill's members in order; each value is picked by selects, so the threads
// of a warp (17 fields per lane) do not split into one path per field.
static_assert(sizeof(DsFill) == (kMetaSecond + 1) * sizeof(int) && offsetof(DsFill, token) == 0 &&
                  offsetof(DsFill, state_out) == kMetaStateOut * sizeof(int) &&
                  offsetof(DsFill, kind) == kMetaKind * sizeof(int) &&
                  offsetof(DsFill, second) == kMetaSecond * sizeof(int),
              "DsFill holds the metadata fields token..second in order");
__device__ inline void write_meta(int* m, int width, const DsFill* f, int n, int draw, bool post,
                                  unsigned long long seed) {
  const int lo = (int)(uint32_t)(seed & 0xFFFFFFFFull), hi = (int)(uint32_t)(seed >> 32);
  for (int i = threadIdx.x; i < width * kMetaFields; i += blockDim.x) {
    const int b = i / kMetaFields, k = i % kMetaFields;
    int v = -1;
    if (b < n) {
      const int stored = reinterpret_cast<const int*>(f + b)[min(k, (int)kMetaSecond)];
      // post rows: kind, first, second, the draw counter and row, the seed, and
      // the single request's parameter slot 0
      const int readout = k == kMetaCycle ? draw : k == kMetaDrawRow ? b : k == kMetaSeedLo ? lo
                        : k == kMetaSeedHi ? hi : k == kMetaReq ? 0 : stored;
      v = k <= kMetaStateOut ? stored : k == kMetaAhead ? 0 : post ? readout : -1;
    }
    m[i] = v;
  }
}

// The state moves in 16-byte pieces (both copies are 16-byte aligned).
static_assert(sizeof(LoopSched) % 16 == 0, "scheduler state must be a whole number of 16-byte pieces");

__device__ inline void load_sched(LoopSched* s, const LoopSched* g) {
  const int n = (int)(sizeof(LoopSched) / 16);
  int4* d = reinterpret_cast<int4*>(s);
  const int4* src = reinterpret_cast<const int4*>(g);
  for (int i = threadIdx.x; i < n; i += blockDim.x) d[i] = __ldcg(src + i);
  __syncthreads();
}

__device__ inline void store_sched(LoopSched* g, const LoopSched* s) {
  __syncthreads();
  const int n = (int)(sizeof(LoopSched) / 16);
  int4* d = reinterpret_cast<int4*>(g);
  const int4* src = reinterpret_cast<const int4*>(s);
  for (int i = threadIdx.x; i < n; i += blockDim.x) d[i] = src[i];
}

// Where the metadata of a cycle's role calls goes: pre, K core records of
// `stride` ints, post; `width` lanes each (unused lanes inactive).
struct LoopMeta {
  int* pre;
  int* core;
  long stride;
  int* post;
  int width;
  int* active;   // live lanes of the pre, core and post calls (a prefix of each)
};

// Start of a cycle (thread 0 has planned it into the shared arrays): write
// the role calls' metadata. A finished request plans no lanes, so its role
// calls do nothing but stream weights.
struct LoopPlan {
  DsFill pre[kLoopMaxLanes], post[kLoopMaxLanes], core[kLoopMaxK * kLoopMaxLanes];
  int n_pre, n_post, n_core, draw;
};

__device__ inline void loop_plan(LoopSched& s, LoopPlan& p) {   // thread 0
  p.n_pre = p.n_post = p.n_core = 0;
  if (!s.done && !s.err) {
    p.n_core = s.gather();
    s.plan(p.pre, p.n_pre, p.core, p.post, p.n_post);
    s.draw_cycle += 1;
  }
  p.draw = s.draw_cycle;
}

__device__ inline void loop_write_meta(const LoopSched& s, const LoopPlan& p, const LoopMeta& m) {
  if (threadIdx.x == 0) {
    m.active[0] = p.n_pre;
    m.active[1] = p.n_core;
    m.active[2] = p.n_post;
  }
  write_meta(m.pre, m.width, p.pre, p.n_pre, p.draw, false, s.seed);
  for (int k = 0; k < s.K; ++k)
    write_meta(m.core + k * m.stride, m.width, p.core + k * kLoopMaxLanes, p.n_core, p.draw, false, s.seed);
  write_meta(m.post, m.width, p.post, p.n_post, p.draw, true, s.seed);
}

// The first cycle's plan.
__global__ void __launch_bounds__(kLoopThreads) loop_plan_kernel(LoopSched* g, LoopMeta m) {
  __shared__ __align__(16) LoopSched s;
  __shared__ LoopPlan p;
  load_sched(&s, g);
  if (threadIdx.x == 0) loop_plan(s, p);
  __syncthreads();
  loop_write_meta(s, p, m);
  store_sched(g, &s);
}

// Launched with programmatic overlap after the post call (its last kernel
// triggers dependents at its start).
// End of a cycle and start of the next: the readout lanes' decisions (in
// readout order: greedy tokens, stride 1, or sampled decision rows, stride 5)
// resolve the pipeline, commit a token to `out` and retain the surviving
// branches' timelines; then the next cycle is planned.
__global__ void __launch_bounds__(kLoopThreads) loop_step_kernel(LoopSched* g, const long long* dec_in, int stride,
                                                                 long long* out, LoopMeta m) {
  __shared__ __align__(16) LoopSched s;
  __shared__ LoopPlan p;
  // the state was written by the previous cycle's step: load it while the
  // post call finishes, then wait for the decisions
  __shared__ long long s_dec_in[kLoopMaxLanes * 5];
  // the next cycle's first kernel may start now: it reads nothing before its
  // own wait, which ends when this kernel has completed
  pdl_launch_dependents();
  load_sched(&s, g);
  pdl_wait();
  // the readouts' decisions, one global round trip for all of them
  if ((int)threadIdx.x < kLoopMaxLanes * stride) s_dec_in[threadIdx.x] = __ldcg(dec_in + threadIdx.x);
  __syncthreads();
  if (threadIdx.x == 0) {
    if (!s.done && !s.err) {
      long long dec[kLoopMaxLanes * 5];
      int j = 0;
      for (int i = 0; i < s.n_lanes; ++i) {
        const bool readout = s.kind_of[s.lanes[i].stage + s.K - 1] >= 0;
        for (int f = 0; f < stride; ++f) dec[i * stride + f] = readout ? s_dec_in[j * stride + f] : -1;
        j += readout;
      }
      s.consume(dec, stride, out);
    }
    loop_plan(s, p);
  }
  __syncthreads();
  loop_write_meta(s, p, m);
  store_sched(g, &s);
}

}  // namespace ls
