/*
 * loopspec_engine.h -- C ABI of the B200-native LoopSpec decode engine
 * (libloopspec_engine.so, built for sm_100a).
 *
 * One engine handle serves one looped model on one GPU. It runs one request
 * at a time through the reference-shaped entry points, like the reference's
 * batch-1 LoopSpec server (sglang_recurrent/server/cli.py:88-89), and up to
 * max_requests together through ls_generate_batch. Plain pointers and sizes only: no
 * torch types cross this boundary. Weight pointers are device pointers owned
 * by the caller; the engine owns its KV pool, timeline mapping table, state
 * banks and workspaces. Every function returns 0 on success or a negative
 * LS_E* code; ls_last_error() returns the message. Calls on one handle must
 * not overlap (single-threaded per handle, stream-ordered inside).
 */
#ifndef LOOPSPEC_ENGINE_H
#define LOOPSPEC_ENGINE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LS_OK 0
#define LS_EINVAL (-1)      /* invalid argument or state                       */
#define LS_ECAPACITY (-2)   /* slots / rows / lanes exhausted (the reference's
                               RuntimeErrors: decode_slots.py:129-134,
                               manager.py:216-217, executor.py:87-93)         */
#define LS_ECUDA (-3)       /* CUDA runtime or driver error                    */
#define LS_EDEVICE (-4)     /* a kernel reported a bounded-wait timeout or a
                               bad index (see ls_last_error)                   */
#define LS_EPIPELINE (-5)   /* scheduler invariant violated (pipeline.py:298-421) */

/* Model families / block layouts (modeling/contracts.py:179-197). */
#define LS_FAMILY_OURO 0
#define LS_FAMILY_RAVEN 1
#define LS_LAYOUT_OURO 0       /* Gemma2 residual flow, sandwich RMSNorm      */
#define LS_LAYOUT_RAVEN_PRE 1  /* Llama pre-norm                              */
#define LS_LAYOUT_OLMO_POST 2  /* OLMo2 post-norm + QK-norm                   */

typedef struct ls_model_cfg {
  int32_t family, layout;
  int32_t hidden, n_heads, n_kv_heads, head_dim, intermediate, vocab;
  int32_t n_pre_layers, n_core_layers, n_post_layers;
  int32_t stages;            /* S: total_ut_steps / mean_recurrence */
  float rope_theta, rms_eps, embed_scale, init_std;
  uint64_t init_seed;        /* Raven position-keyed hidden init */
  int32_t qk_norm, adapter_bias, tie_embeddings;
} ls_model_cfg;

/* Schedule and capacities. step_size = K (--first), second_step = X =
 * D / K (--second D), 0 = no q2 (pipeline.py:124-139). */
typedef struct ls_sched_cfg {
  int32_t step_size, second_step;
  int32_t max_context;       /* max positions per timeline (prompt + output) */
  int32_t max_prompt;        /* longest prompt accepted by ls_prefill        */
  int32_t kv_slots;          /* KV token slots per attention layer (0: auto) */
  int32_t request_rows;      /* timeline mapping rows (0: auto)              */
  int32_t use_graphs;        /* capture one CUDA graph per (role, width)     */
  int32_t use_pdl;           /* programmatic dependent launch between kernels */
  int32_t max_requests;      /* requests ls_generate_batch serves together (0: 1);
                                request_rows / kv_slots size each of them      */
  int32_t device_loop;       /* 1: ls_generate runs a LoopSpec request, greedy
                                or sampled, as captured graphs of 8 cycles with
                                the scheduler on the GPU (no host round trip
                                between cycles), when the schedule fits (<= 16
                                live lanes, S <= 8, K <= 8), one request is
                                configured, kv_slots is 0 and its KV pool stays
                                within 24 GB; otherwise, and for streaming
                                callbacks, tensor parallelism or batches, the
                                host drives each cycle                           */
} ls_sched_cfg;

/* Counters of sglang_recurrent/loopspec/executor.py:35-45 plus timing. */
typedef struct ls_stats {
  int64_t pipeline_cycles, pre_rows, recurrent_rows, post_rows;
  int64_t verified_proposals, first_rejections, second_verifications;
  int64_t second_acceptances, second_rejections;
  int64_t decode_tokens;     /* committed tokens after the first */
  double decode_device_ms;   /* CUDA-event time of the decode loop            */
  double decode_host_s;      /* host clock, after first token to last commit  */
  double prefill_device_ms;
  int64_t h2d_bytes;         /* host->device bytes copied for the request       */
  int64_t d2h_bytes;         /* device->host bytes copied for the request       */
  int64_t decode_kernel_launches; /* engine kernels launched by the decode loop */
  /* Work of the decode loop, for the bytes-moved roofline: */
  int64_t pre_calls;         /* pre role calls that ran prelude layers        */
  int64_t core_calls;        /* core role calls (one per core iteration)      */
  int64_t core_kv_positions; /* sum over core lanes of the timeline length
                                each attended (KV rows read per core layer)   */
  int64_t post_calls;        /* post role calls that ran the lm_head          */
  int64_t host_syncs;        /* times the decode loop waited for the GPU      */
} ls_stats;

typedef struct ls_engine ls_engine;

/* Create an engine on `device` (replaces make_loopspec_runner,
 * server/loopspec_runner.py:118-195). */
int ls_create(const ls_model_cfg* model, const ls_sched_cfg* sched, int device, ls_engine** out);

/* Borrow one bf16 weight (device pointer) under the reference's internal
 * parameter name (RecurrentServingModel.load_weights, modeling/serving.py:142-182;
 * names after ouro.py:19-34 / raven.py:221-255 mapping, packed qkv_proj and
 * gate_up_proj). dtype: 0 = bf16 (the only accepted type). */
int ls_load_weight(ls_engine* eng, const char* name, const void* dptr, int dtype,
                   const int64_t* shape, int ndim);

/* Validate the weight set, allocate pools and build TMA descriptors. */
int ls_finalize(ls_engine* eng);

/* Tensor parallelism (one process per GPU). Each rank creates its engine
 * from its shard: n_heads, n_kv_heads and intermediate divided by the rank
 * count, q/k/v rows and gate/up rows of its heads and columns, o_proj and
 * down_proj columns of the same, q_norm / k_norm entries of its heads, all
 * other weights whole. After ls_finalize, ls_tp_init allocates the rank's
 * exchange region and writes LS_TP_HANDLE_BYTES describing it (CUDA IPC
 * handle, PCI bus id, layout size); the caller gathers every rank's bytes in
 * rank order (any host collective) and passes them to ls_tp_attach. From
 * then on every rank must make the same calls with the same arguments: the
 * layers add all ranks' O / down partials and QK-norm sums in rank order
 * over NVLink, so all ranks compute identical rows and decisions. A peer
 * that stops publishing makes the waiting ranks fail with LS_EDEVICE after a
 * bounded wait. Ranks must be on distinct GPUs, and ls_tp_init must precede
 * the first role call. The reference
 * rejects tensor parallelism for LoopSpec (cli.py:97-108); the target is
 * TP-N greedy output equal to TP-1 output. */
#define LS_TP_HANDLE_BYTES 128
int ls_tp_init(ls_engine* eng, int rank, int ranks, void* handle_out);
int ls_tp_attach(ls_engine* eng, const void* handles);

/* Reset request state and prefill every timeline of the prompt (pre, all S
 * core depths, each post endpoint with attention), then pick the first token
 * greedily (RecurrentRequest.prefill request.py:111-192 and
 * _sample_first_token executor.py:161-182). out_logits: optional host
 * float[vocab] receiving the final-depth logits of the last prompt token. */
int ls_prefill(ls_engine* eng, const int64_t* prompt, int n_prompt, float* out_logits,
               int64_t* first_token);

/* Sampling settings of the next request(s) (the reference's request-level
 * {temperature, top_k, top_p} and sampling_seed, server/loopspec_scheduler.py:
 * 316-329). Greedy iff top_k == 1 or temperature == 0 (the default). Sampled
 * decisions follow sampling/policy.py: top-p / top-k filtered softmax, q1 draw,
 * q2 conditional residual, final verification and the rejection fallback, all
 * on the GPU; uniforms come from Philox4x32-10 keyed by `seed`. */
int ls_set_sampling(ls_engine* eng, float temperature, int top_k, float top_p, uint64_t seed);

/* One pipeline cycle over `n_lanes` lanes (LosslessLoopSpecExecutor.forward,
 * executor.py:293-367, without the host resolve step): pre for stage-0 lanes,
 * K core iterations for all lanes, post + decision for lanes whose last
 * iteration is a q1/q2/final readout. lanes: int64 [n_lanes][8] =
 * (stage, index, token, branch, parent_branch or -1, state_slot, q1 token or
 * -1, q2 token or -1). out_decisions: int64 [n_lanes][5] per readout lane:
 * greedy -> (argmax, 0, 0, 0, 0); sampling -> (token, proposed,
 * accepted_code, q1_rejected, q2_rejected) as policy.py:197-283; other lanes
 * (-1, 0, 0, 0, 0). out_logits: optional host float [n_lanes][vocab] (rows of
 * non-readout lanes are left untouched). Synchronises once (readback). */
int ls_cycle(ls_engine* eng, const int64_t* lanes, int n_lanes, int64_t* out_decisions,
             float* out_logits);

/* Keep the timelines of the surviving lanes and release the rest
 * (BranchManager.retain_branches, branching/manager.py:453-482).
 * branch_ids / parent_ids: int64 [n] (parent -1 for none); n = 0 ends the
 * request and frees every branch. */
int ls_retain(ls_engine* eng, const int64_t* branch_ids, const int64_t* parent_ids, int n);

/* Whole request natively: prefill, first token, then the LoopSpec pipeline
 * (mode 0: continue_pipelined pipeline.py:254-423 with greedy decisions
 * decisions.py:136-184) or plain autoregressive decoding (mode 1: one token
 * per step through pre, S core iterations and post, serving.py:216-239).
 * stop_token < 0 disables EOS stopping. out_ids: int64 [max_new_tokens]. */
int ls_generate(ls_engine* eng, const int64_t* prompt, int n_prompt, int max_new_tokens,
                int mode, int64_t stop_token, int64_t* out_ids, int* n_out, ls_stats* stats);

/* ls_generate with a commit callback: after every commit (the first token
 * included) on_commit(user, ids, n) receives the whole committed output so
 * far, as the reference's should_stop does (loopspec_scheduler.py:331-346,
 * pipeline.py:64); a nonzero return ends the request there. This carries
 * streaming at interval 1 and caller-side stop rules; stop_token still ends
 * at EOS. The callback runs on the calling thread between GPU steps. */
typedef int (*ls_commit_fn)(void* user, const int64_t* ids, int n);
int ls_generate_stream(ls_engine* eng, const int64_t* prompt, int n_prompt, int max_new_tokens,
                       int mode, int64_t stop_token, ls_commit_fn on_commit, void* user,
                       int64_t* out_ids, int* n_out, ls_stats* stats);

/* Several requests decoded together (no counterpart in the reference, whose
 * LoopSpec server runs one request at a time, server/cli.py:88-89). Each
 * request is prefilled in turn, then every cycle runs one pre, K core and one
 * post call over the lanes of all running requests (mode 0: one
 * continue_pipelined per request, pipeline.py:254-423; mode 1: one
 * autoregressive step per running request). Each request keeps its own branch
 * timelines, state slots, random-stream cycle and seed (seeds[i], or the
 * ls_set_sampling seed + i when seeds is NULL), and every kernel computes a
 * lane's numbers independently of the other lanes of its call, so request i
 * commits exactly what it commits alone with the same seed. prompts: the
 * n_requests prompts back to back, prompt_lens[i] tokens each (n_requests <=
 * max_requests). out_ids: int64 [n_requests][max_new_tokens]; n_out: int32
 * [n_requests]. per_request (optional, [n_requests]): each request's scheduler
 * counters and tokens, with the batch's decode time; total (optional): their
 * sums, the batch's work counters, copy volumes and decode time. */
int ls_generate_batch(ls_engine* eng, const int64_t* prompts, const int32_t* prompt_lens,
                      int n_requests, int max_new_tokens, int mode, int64_t stop_token,
                      const uint64_t* seeds, int64_t* out_ids, int32_t* n_out,
                      ls_stats* per_request, ls_stats* total);

/* ls_generate_batch with each request's own sampling parameters, so greedy
 * and sampled requests share a batch: request i decodes with temperature[i],
 * top_k[i], top_p[i] (greedy iff temperature == 0 or top_k == 1, the
 * reference server's rule, server/loopspec_scheduler.py:316-329) and draws
 * from seeds[i] (required). Each request commits what it commits alone with
 * the same parameters and seed. The engine's own ls_set_sampling state is
 * unchanged afterwards. Replaces, per request, the SamplingParams the
 * reference's server takes with each /generate call (cli.py:88-89 serves one
 * at a time). */
int ls_generate_batch_sampling(ls_engine* eng, const int64_t* prompts, const int32_t* prompt_lens,
                               int n_requests, int max_new_tokens, int mode, int64_t stop_token,
                               const uint64_t* seeds, const float* temperature,
                               const int32_t* top_k, const float* top_p, int64_t* out_ids,
                               int32_t* n_out, ls_stats* per_request, ls_stats* total);

/* The native scheduler loop of ls_generate mode 0 (continue_pipelined,
 * pipeline.py:254-423, with greedy resolve decisions.py:136-184 and the
 * executor's state-slot pool and counters executor.py:76-107,239-290),
 * driven by host callbacks instead of the GPU: `decide` returns the token a
 * readout of lane (index, input token) yields (kind 0 q1, 1 q2, 2 final);
 * `on_cycle` sees each cycle's lanes as int64 [n][7] = (stage, index,
 * token, branch, parent|-1, origin_stage|-1, state_slot); `on_retain` sees
 * each retention as int64 [n][2] = (branch, parent|-1) plus the accepted
 * stage (-1 for none). Needs no GPU. */
typedef int64_t (*ls_decide_fn)(void* user, int64_t index, int64_t token, int32_t kind);
typedef void (*ls_cycle_fn)(void* user, const int64_t* lanes, int32_t n);
typedef void (*ls_retain_fn)(void* user, const int64_t* pairs, int32_t n, int32_t accepted_stage);
int ls_pipeline_simulate(int stages, int step_size, int second_step, int64_t first_token,
                         int max_new_tokens, int64_t stop_token, ls_decide_fn decide,
                         ls_cycle_fn on_cycle, ls_retain_fn on_retain, void* user,
                         int64_t* out_ids, int* n_out, ls_stats* stats);

/* ls_pipeline_simulate running the scheduler of the device-resident decode
 * loop (the fixed-size state that one GPU thread runs between the role calls
 * of a cycle; no reference counterpart beyond the loop it restates) compiled
 * for the host: same arguments, callbacks and results. Needs no GPU. */
int ls_device_loop_simulate(int stages, int step_size, int second_step, int64_t first_token,
                            int max_new_tokens, int64_t stop_token, ls_decide_fn decide,
                            ls_cycle_fn on_cycle, ls_retain_fn on_retain, void* user,
                            int64_t* out_ids, int* n_out, ls_stats* stats);

/* Time one role call of `n_lanes` synthetic lanes (role 0 pre, 1 core, 2
 * post) `iters` times with CUDA events on the engine stream, after a
 * prefill; returns the average device milliseconds per call. Used by the
 * benchmark's roofline report. context_len sets every lane's position. */
int ls_time_role(ls_engine* eng, int role, int n_lanes, int context_len, int iters,
                 double* avg_ms);

/* Time one GEMM of the core layer 0 (which: 0 qkv, 1 o, 2 gate_up, 3 down,
 * 4 lm_head) over n_lanes lanes, `iters` launches; average device ms. */
int ls_time_gemm(ls_engine* eng, int which, int n_lanes, int iters, double* avg_ms);

/* Time every core GEMM of one recurrent iteration (qkv, o, gate_up, down
 * for each core layer, one launch each) over n_lanes lanes, `iters` sweeps
 * back to back with CUDA events on the engine stream. The sweep streams all
 * core weights (larger than L2), so no launch reads another's weights from
 * L2. Returns the average launch time and the average algorithmic bytes of
 * one launch (weights + activation rows read + fp32 partials written). */
int ls_time_core_gemms(ls_engine* eng, int n_lanes, int iters, double* avg_launch_ms,
                       double* bytes_per_launch);

/* Number of kernels one role call of n_lanes launches. */
int ls_role_kernel_count(ls_engine* eng, int role, int n_lanes, int* count);

/* Run one GEMM of core layer 0 (which: 0 qkv, 1 o, 2 gate_up, 3 down,
 * 4 lm_head, 5 Raven adapter) on host activations x (fp32 [n][K], fed as a
 * bf16 hi/lo pair per lane like every engine GEMM) and return the
 * split-summed fp32 result [n][rows], for kernel tests. */
int ls_debug_gemm(ls_engine* eng, int which, int n_lanes, const float* x, float* out);
int ls_gemm_splits(ls_engine* eng, int which, int* splits, int* rows, int* k);

/* Device pointer of the engine's KV pool (K then V, each
 * [attn_layers][kv_slots][n_kv_heads*head_dim] bf16), for tests. */
int ls_debug_kv(ls_engine* eng, void** k_pool, void** v_pool, int* kv_slots, int* attn_layers);

/* Failure-detection test of the tensor-parallel exchange on one GPU: after
 * ls_tp_init(eng, rank, 2, ...), attach a zeroed region of this GPU as the
 * other rank's. Its flags never rise, so the first exchange waits wait_ms,
 * records "tensor-parallel peer wait timed out" and later exchanges give up
 * at once; the call then fails with LS_EDEVICE and the context stays usable. */
int ls_debug_tp_silent_peer(ls_engine* eng, int wait_ms);

/* Branch-timeline paged decode attention of one layer, standalone (the
 * engine's attention kernel; replaces SGLang's Triton decode attention as the
 * reference drives it through req_to_token rows, cuda_graph.py:361-394).
 * Lane i has one query q[i] (fp32 [n_heads*head_dim], RoPE applied) and
 * attends to positions 0..lane_lens[i]-1 of mapping row lane_rows[i]:
 * position j's K/V live in slot map[row*max_context + j] of k_pool / v_pool
 * (bf16 [n_slots][n_kv_heads*head_dim]). Forked timelines share slots.
 * out: fp32 [n_lanes][n_heads*head_dim]. All pointers are device memory
 * (lane_rows / lane_lens int32 [n_lanes]). workspace: device scratch of at
 * least ls_decode_attention_workspace_bytes() bytes, 256-byte aligned.
 * Runs on `stream` (cudaStream_t, NULL = legacy default) and waits for it.
 * Out-of-range rows, lengths or slots are skipped and reported as LS_EDEVICE.
 * Handle-less: errors are read with ls_last_error(NULL). */
size_t ls_decode_attention_workspace_bytes(int n_lanes, int n_heads, int n_kv_heads, int head_dim,
                                           int max_context);
int ls_decode_attention(const float* q, const void* k_pool, const void* v_pool, const int32_t* map,
                        const int32_t* lane_rows, const int32_t* lane_lens, int n_lanes, int n_heads,
                        int n_kv_heads, int head_dim, int n_slots, int n_rows, int max_context,
                        void* workspace, size_t workspace_bytes, float* out, void* stream);

/* Allocation-free ls_decode_attention (no counterpart in the reference).
 * For callers that cannot call cudaMalloc (code inside an allocator or
 * memory-pool hook, runtimes that reserve all device memory up front,
 * processes that forbid device allocation after start-up). Same arguments
 * and result as ls_decode_attention minus the workspace: the scratch is a
 * fixed 4 MiB array inside the library (ls_decode_attention_noalloc_limit()),
 * held on every GPU that loads the library until exit. Shapes whose scratch
 * (about n_lanes * n_heads * ceil(max_context/128) * (head_dim + 2) * 4
 * bytes: one partial per 128-position chunk) exceeds it are rejected with
 * LS_ECAPACITY. The first call on a device looks up the array's device
 * address and keeps it for the life of the process (a device reset would
 * make it stale), so make that first call before any stream capture. Like
 * ls_decode_attention, each call waits for `stream` to finish before it
 * returns. All calls on a device share the array: the call clears what must
 * start at zero, later calls overwrite the rest, and calls that overlap on
 * the GPU race. Calls no cudaMalloc, cudaFree or allocating library
 * routine. */
int ls_decode_attention_noalloc(const float* q, const void* k_pool, const void* v_pool,
                                const int32_t* map, const int32_t* lane_rows,
                                const int32_t* lane_lens, int n_lanes, int n_heads, int n_kv_heads,
                                int head_dim, int n_slots, int n_rows, int max_context, float* out,
                                void* stream);
size_t ls_decode_attention_noalloc_limit(void);

int ls_destroy(ls_engine* eng);
const char* ls_last_error(ls_engine* eng);
const char* ls_version(void);

#ifdef __cplusplus
}
#endif

#endif /* LOOPSPEC_ENGINE_H */
