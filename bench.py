#!/usr/bin/env python
"""LoopSpec decode benchmark (the Ouro-1.4B batch-1 configuration by default).

Workload: Ouro-1.4B architecture, random init (seed 0), bf16 weights, batch 1,
a 512-token prompt of uniform-random ids, 1024 greedy new tokens, LoopSpec
first=1 second=2 (K=1, X=2), with the autoregressive path timed beside it.
One step = one request through the public API (`generate_loopspec`).

value   decode tokens/s (tokens after the first, as the reference's
        generation_metrics, server/metrics.py:21-30) = sum of decode tokens of
        all ranks / max over ranks of CUDA-event decode time; inputs already
        resident in HBM.
e2e     the same tokens / host wall time of the whole generate_loopspec call
        (prompt upload, prefill, decode, readbacks), max over ranks.
--impl reference   the reference algorithm's CPU implementation (the oracle
        port: reference scheduler restated + fp32 model roles) on the host
        cores, on a bounded sample of the same workload.
Multi-GPU: one process per GPU, independent request replicas (weak scaling).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

from loopspec_b200 import roofline  # noqa: E402
from loopspec_b200.config import get_config  # noqa: E402
from loopspec_b200.schedule import PipelineSchedule, accept_length  # noqa: E402

METRIC = "decode tokens/s/GPU (bs=1, 1-8 B200), LoopSpec vs AR speedup, mean accepted len"
UNIT = "tokens/s"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=3)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="engine", choices=["engine", "reference"])
    p.add_argument("--config", default="ouro-1.4b")
    p.add_argument("--prompt", type=int, default=512)
    p.add_argument("--new-tokens", type=int, default=1024)
    p.add_argument("--first", type=int, default=1)
    p.add_argument("--second", type=int, default=2)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--synthetic-accept", type=float, default=0.05,
                   help="post-norm gain of the separately reported high-acceptance run (0: skip)")
    p.add_argument("--temperature", type=float, default=0.0,
                   help="> 0: sampled decoding (with --top-p / --top-k) instead of greedy")
    p.add_argument("--top-p", type=float, default=1.0)
    p.add_argument("--top-k", type=int, default=0)
    p.add_argument("--seed", type=int, default=1234, help="sampling seed of request i is seed + i")
    p.add_argument("--batch", type=int, default=0,
                   help="> 0: serve this many requests together per step (ls_generate_batch), split "
                        "over the ranks; prompt lengths uniform in [--prompt-min, --prompt]")
    p.add_argument("--prompt-min", type=int, default=0,
                   help="shortest prompt of a --batch step (0: every prompt has --prompt tokens)")
    p.add_argument("--mixed", action="store_true",
                   help="with --batch and --temperature: every other request decodes greedily "
                        "(per-request parameters, as config 5 mixes greedy and top-p requests)")
    p.add_argument("--host-loop", action="store_true",
                   help="run LoopSpec cycles from the host (one sync per cycle) instead of the "
                        "device-resident loop")
    p.add_argument("--tp", action="store_true",
                   help="under torchrun: one request split over the ranks by tensor parallelism "
                        "(heads and MLP columns; strong scaling) instead of one replica per GPU")
    return p.parse_args()


def decode_mode(args):
    if args.temperature <= 0:
        return "greedy"
    return f"sampled T={args.temperature} top_p={args.top_p} top_k={args.top_k} seed={args.seed}+i"


def sampling_of(args):
    """None (greedy) or the request sampling dict of generate_loopspec."""
    if args.temperature <= 0:
        return None
    return {"temperature": args.temperature, "top_p": args.top_p, "top_k": args.top_k}


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), \
        int(os.environ.get("LOCAL_RANK", 0))


def make_prompt(cfg, n, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, cfg.vocab, (n,), generator=g).tolist()


def schedule_for(cfg, args):
    from loopspec_b200.config import parse_loopspec_flags
    K, X = parse_loopspec_flags(cfg.stages, args.first, args.second)
    return PipelineSchedule(cfg.stages, K, X)


class Clocks:
    """nvidia-smi sampling during the timed region (one GPU)."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu):
        self.gpu = gpu
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        self.proc.wait(timeout=10)
        rows = []
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) >= 9:
                rows.append(f)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(rows)}


L2_BYTES = 126 * 2**20   # B200 L2


def l2_note(cfg):
    """How the timed steps relate to L2: each core iteration streams this
    rank's core weights, larger than L2 for every shipped config but the tiny ones."""
    w = cfg.core_weight_bytes()
    if w > L2_BYTES:
        return f"inputs larger than L2 ({w / 1e9:.2f} GB of core weights per iteration on each GPU)"
    return f"core weights ({w / 1e6:.1f} MB per iteration) fit in L2; no flush between steps"


def cpu_baseline(cfg, sch, args, threads):
    """The oracle (reference algorithm, CPU, fp32) on a bounded sample."""
    from oracle.executor import generate_loopspec_oracle
    from oracle.model import OracleModel
    from loopspec_b200.weights import init_random_weights
    torch.set_num_threads(threads)
    w = init_random_weights(cfg, 0, device="cpu", dtype=torch.float32)
    model = OracleModel(cfg.as_dict(), w)
    del w
    prompt = make_prompt(cfg, 8, 7)
    n_new = 5
    t0 = time.perf_counter()
    ids, st = generate_loopspec_oracle(model, sch, prompt, n_new)
    dt = time.perf_counter() - t0
    # oracle processes prompt tokens one at a time through all depths; count
    # decode tokens only, against the whole sample's time (conservative)
    return {"value": round(st["decode_tokens"] / dt, 4), "unit": UNIT, "cores": threads,
            "kind": "port",
            "sample": f"{cfg.name} fp32 oracle, 8-token prompt, {n_new} LoopSpec "
                      f"K={sch.step_size} X={sch.second_step} greedy tokens, time incl. prefill"}


def reference_arm(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    cfg = get_config(args.config)
    sch = schedule_for(cfg, args)
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    from oracle.executor import generate_loopspec_oracle
    from oracle.model import OracleModel
    from loopspec_b200.weights import init_random_weights
    w = init_random_weights(cfg, 0, device="cpu", dtype=torch.float32)
    model = OracleModel(cfg.as_dict(), w)
    del w
    n_prompt, n_new = 8, 4
    times, toks = [], []
    for i in range(args.warmup + args.steps):
        prompt = make_prompt(cfg, n_prompt, 100 + i)
        t0 = time.perf_counter()
        ids, st = generate_loopspec_oracle(model, sch, prompt, n_new)
        dt = time.perf_counter() - t0
        if i >= args.warmup:
            times.append(dt)
            toks.append(st["decode_tokens"])
    value = sum(toks) / sum(times)
    sample = (f"{cfg.name} fp32 oracle on {threads} host threads: {n_prompt}-token prompt, "
              f"{n_new} greedy LoopSpec tokens per step (time incl. the prompt pass)")
    line = {"metric": METRIC, "value": round(value, 4), "unit": UNIT, "impl": "reference",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(1e3 * sum(times) / len(times), 1), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"{cfg.name} LoopSpec first={args.first} second={args.second} "
                                   f"greedy (bounded CPU sample)", "global_batch": 1},
            "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": threads,
                             "kind": "port", "sample": sample},
            "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def tp_block(args, rank, world, local, dist):
    """Tensor parallelism beside the replica run (N > 1): the largest Raven
    model (Raven-OLMo, LoopSpec 2:8) split over all N ranks by heads and MLP
    columns, against the same work on one GPU (rank 0): one short greedy
    request, then a batch of 8 (4 greedy, 4 top-p 0.9 requests with their own
    parameters, as config 5 mixes them). Bounded: every rank builds its shard
    first and all ranks agree that every engine exists before any kernel
    runs; a failure is reported in the block instead of ending the
    benchmark."""
    from loopspec_b200.engine import Engine
    from loopspec_b200.executor import generate_loopspec, generate_loopspec_batch
    from loopspec_b200.tp import shard_config, shard_weights
    from loopspec_b200.weights import init_random_weights
    cfg = get_config("raven-olmo")
    sch = PipelineSchedule(cfg.stages, 2, 4)
    n_prompt, n_new, n_batch = 64, 64, 8
    prompts = [make_prompt(cfg, n_prompt, 77 + i) for i in range(n_batch)]
    samp = [None if i % 2 == 0 else {"temperature": 1.0, "top_k": 0, "top_p": 0.9} for i in range(n_batch)]
    seeds = [4242 + i for i in range(n_batch)]
    out = {"model": cfg.name, "ranks": world, "schedule": "LoopSpec first=2 second=8",
           "prompt": n_prompt, "new_tokens": n_new}

    def decode(eng, n_req):
        if n_req == 1:
            generate_loopspec(eng, prompts[0], n_new)                  # warm-up / capture
            ids, st = generate_loopspec(eng, prompts[0], n_new)
            return [ids], st["decode_tokens"] / (st["decode_device_ms"] / 1e3)
        generate_loopspec_batch(eng, prompts, n_new, sampling=samp, seeds=seeds)
        ids, _, tot = generate_loopspec_batch(eng, prompts, n_new, sampling=samp, seeds=seeds)
        return ids, tot["decode_tokens"] / (tot["decode_device_ms"] / 1e3)

    def measure(n_req):
        res = {}
        eng = None
        ok = True
        try:
            w = init_random_weights(cfg, 0, device=f"cuda:{local}", dtype=torch.bfloat16)
            eng = Engine(shard_config(cfg, world), sch, shard_weights(w, cfg, rank, world), device=local,
                         max_context=256, max_prompt=n_prompt, max_requests=n_req)
            del w
            handle = eng.tp_init(rank, world)
        except Exception as ex:   # noqa: BLE001 - reported, the replica line still prints
            ok, handle, res["error"] = False, b"", repr(ex)[:300]
        got = [None] * world
        dist.all_gather_object(got, (ok, handle))
        ids = None
        if all(g[0] for g in got):
            try:
                eng.tp_attach([g[1] for g in got])
                ids, rate = decode(eng, n_req)
                res["tp_tok_s"] = round(rate, 2)
            except Exception as ex:   # noqa: BLE001
                res["error"] = repr(ex)[:300]
        ms = torch.tensor([res.get("tp_tok_s", 0.0)], dtype=torch.float64, device="cuda")
        dist.all_reduce(ms, op=dist.ReduceOp.MIN)                     # slowest rank
        dist.barrier()      # no rank releases its exchange region while a peer may read it
        if eng is not None:
            eng.close()
        if rank == 0 and "error" not in res:
            res["tp_tok_s"] = round(float(ms.item()), 2)
            w1 = init_random_weights(cfg, 0, device=f"cuda:{local}", dtype=torch.bfloat16)
            one = Engine(cfg, sch, w1, device=local, max_context=256, max_prompt=n_prompt,
                         max_requests=n_req)
            ids1, rate1 = decode(one, n_req)
            one.close()
            res["single_gpu_tok_s"] = round(rate1, 2)
            res["tokens_equal_single_gpu"] = ids1 == ids
            res["speedup_vs_single_gpu"] = round(res["tp_tok_s"] / res["single_gpu_tok_s"], 3)
        dist.barrier()
        return res

    out.update(measure(1))
    out["batch8_mixed"] = measure(n_batch)
    return out


def engine_arm(args):
    from loopspec_b200.engine import Engine
    from loopspec_b200.executor import generate_autoregressive, generate_loopspec
    from loopspec_b200.weights import init_random_weights

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))

    def barrier():
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()

    def max_over_ranks(x):
        if dist is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def sum_over_ranks(x):
        if dist is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return float(t.item())

    cfg = get_config(args.config)
    sch = schedule_for(cfg, args)
    weights = init_random_weights(cfg, 0, device=f"cuda:{local}", dtype=torch.bfloat16)
    max_ctx = args.prompt + args.new_tokens + 64
    tp = args.tp and world > 1
    if tp:
        from loopspec_b200.tp import make_tp_engine
        eng = make_tp_engine(cfg, sch, weights, rank, world, device=local, max_context=max_ctx,
                             max_prompt=args.prompt)
        del weights
    else:
        eng = Engine(cfg, sch, weights, device=local, max_context=max_ctx, max_prompt=args.prompt,
                     device_loop=not args.host_loop)

    def prompt_of(i):
        # under tensor parallelism every rank serves the same request
        return make_prompt(cfg, args.prompt, (0 if tp else 1000 * rank) + i)

    samp = sampling_of(args)
    for i in range(args.warmup):
        generate_loopspec(eng, prompt_of(i), args.new_tokens, sampling=samp, seed=args.seed + i)
    barrier()
    clocks = Clocks(local)
    clocks.start()
    dec_tok = dec_ms = wall = 0.0
    h2d = d2h = 0
    agg = None
    useful = 0
    first_ids = None
    for i in range(args.steps):
        t0 = time.perf_counter()
        ids, st = generate_loopspec(eng, prompt_of(args.warmup + i), args.new_tokens, sampling=samp,
                                    seed=args.seed + args.warmup + i)
        wall += time.perf_counter() - t0
        if first_ids is None:
            first_ids = ids
        useful += roofline.useful_bytes(eng.cfg, st["decode_tokens"], args.prompt)
        dec_tok += st["decode_tokens"]
        dec_ms += st["decode_device_ms"]
        h2d += st["h2d_bytes"] + 8 * args.prompt
        d2h += st["d2h_bytes"]
        agg = st if agg is None else {k: agg[k] + st[k] for k in st}
    barrier()
    clk = clocks.stop()
    dec_s_max = max_over_ranks(dec_ms / 1e3)
    wall_max = max_over_ranks(wall)
    tok_all = dec_tok if tp else sum_over_ranks(dec_tok)
    new_all = args.steps * args.new_tokens if tp else sum_over_ranks(args.steps * args.new_tokens)
    value = tok_all / dec_s_max
    e2e = new_all / wall_max

    # Separately reported: the same request on weights whose post-norm gains
    # are scaled down (small recurrent updates, so early readouts agree with the
    # final one). Uniform random weights reject every draft; this shows what the
    # pipeline does when drafts are accepted. Not the headline value.
    synth = None
    if args.synthetic_accept and rank == 0 and not tp:
        w2 = init_random_weights(cfg, 0, device=f"cuda:{local}", dtype=torch.bfloat16)
        for k in w2:
            if k.endswith(("post_attention_layernorm.weight", "post_feedforward_layernorm.weight")):
                w2[k].mul_(args.synthetic_accept)
        eng2 = Engine(cfg, sch, w2, device=local, max_context=max_ctx, max_prompt=args.prompt,
                      device_loop=not args.host_loop)
        generate_loopspec(eng2, prompt_of(0), args.new_tokens)
        _, s_ls = generate_loopspec(eng2, prompt_of(1), args.new_tokens)
        _, s_ar = generate_autoregressive(eng2, prompt_of(1), args.new_tokens)
        ls_tps = s_ls["decode_tokens"] / (s_ls["decode_device_ms"] / 1e3)
        ar_tps = s_ar["decode_tokens"] / (s_ar["decode_device_ms"] / 1e3)
        synth = {"init": f"post-norm weights x{args.synthetic_accept}", "loopspec_tok_s": round(ls_tps, 2),
                 "ar_tok_s": round(ar_tps, 2), "speedup_vs_ar": round(ls_tps / ar_tps, 3),
                 "mean_accept_len": round(accept_length(s_ls, sch), 4),
                 "first_rejections": int(s_ls["first_rejections"]),
                 "decode_tokens": int(s_ls["decode_tokens"])}
        eng2.close()
        del w2

    # autoregressive beside it, on the first timed request's prompt: greedy
    # LoopSpec must commit exactly the AR tokens
    ar_ids, ar_st = generate_autoregressive(eng, prompt_of(args.warmup), args.new_tokens, sampling=samp,
                                            seed=args.seed + args.warmup)
    ar_tok_s = ar_st["decode_tokens"] / (ar_st["decode_device_ms"] / 1e3)
    ar_gbs = roofline.decode_bytes(eng.cfg, ar_st) / (ar_st["decode_device_ms"] / 1e3) / 1e9
    greedy_equal_ar = (list(first_ids) == list(ar_ids)) if samp is None else None

    # roofline of the dominant kernel: the tcgen05 GEMM, over a core-weight sweep
    lanes = max(1, round(agg["recurrent_rows"] / max(agg["pipeline_cycles"], 1) / sch.step_size))
    launch_ms, launch_bytes = eng.time_core_gemms(lanes, iters=5)
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
        peak_gbs, peak_src = float(peaks["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        peak_gbs, peak_src = 6650.0, "fallback"
    achieved = launch_bytes / (launch_ms / 1e3) / 1e9
    # DRAM traffic per launch: an ncu capture (dram__bytes_read/write.sum) of the
    # layer-0 QKV, O, gate_up and down projections of a 4-lane Ouro-1.4B core call
    # in their decode form read 103.234 MB and wrote 0 B for 103.203 MB of
    # algorithmic bytes (ratio 1.0003: no tile read twice, the split planes stay in
    # L2); scaled to this sweep's average launch.
    traffic = launch_bytes * (103.234 / 103.203)
    # per rank: under tensor parallelism its shard of the core and its KV heads.
    # All bytes moved (rejected lanes included), and the AR bytes of the
    # committed tokens (the useful work), over the same decode time.
    decode_bytes = roofline.decode_bytes(eng.cfg, agg)
    decode_gbs = decode_bytes / (dec_ms / 1e3) / 1e9
    useful_gbs = useful / (dec_ms / 1e3) / 1e9

    tp_info = tp_block(args, rank, world, local, dist) if dist is not None and not tp else None

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(1e3 * wall_max / args.steps, 1),
            "higher_is_better": True, "scaling": "strong" if tp else "weak", "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (uniform-random prompt ids, random-init weights seed 0)",
            "config": {"workload": f"{cfg.name} LoopSpec first={args.first} second={args.second} "
                                   f"{decode_mode(args)}, prompt {args.prompt}, {args.new_tokens} new tokens",
                       "global_batch": 1 if tp else world, "seq_len": args.prompt + args.new_tokens,
                       "parallelism": f"tp{world}" if tp else f"replicas x{world}",
                       "l2": l2_note(eng.cfg)},
            "loopspec_tok_s": round(value if tp else value / world, 2),
            "ar_tok_s": round(ar_tok_s, 2),
            "speedup_vs_ar": round((value if tp else value / world) / ar_tok_s, 3),
            "mean_accept_len": round(accept_length(agg, sch), 4),
            "counters": {k: int(agg[k]) for k in ("pipeline_cycles", "pre_rows", "recurrent_rows",
                                                  "post_rows", "verified_proposals",
                                                  "first_rejections", "second_verifications",
                                                  "second_acceptances", "second_rejections",
                                                  "decode_tokens", "pre_calls", "core_calls",
                                                  "core_kv_positions", "post_calls", "host_syncs")},
            "decode_device_s": round(dec_ms / 1e3, 4),
            "roofline": {"bound": "hbm", "kernel": "gemm_tc_kernel (core weight sweep)",
                         "achieved": round(achieved, 1), "peak": peak_gbs, "unit": "GB/s",
                         "frac": round(achieved / peak_gbs, 4), "peak_source": peak_src,
                         "traffic": round(traffic),
                         "traffic_source": "ncu dram__bytes_read+write of one layer's four core GEMMs "
                                           "(4 lanes), ratio to their algorithmic bytes applied to "
                                           "this sweep",
                         "lanes": lanes,
                         "bytes_per_launch": round(launch_bytes),
                         "avg_launch_us": round(launch_ms * 1e3, 3)},
            "decode_roofline": {"achieved": round(decode_gbs, 1), "peak": peak_gbs,
                                "unit": "GB/s", "frac": round(decode_gbs / peak_gbs, 4),
                                "bytes": round(decode_bytes),
                                "bytes_formula": "core_calls*W_core + pre_calls*W_pre + "
                                                 "post_calls*(W_post+W_lm) + (core_kv_positions + "
                                                 "recurrent_rows)*KV_row (from counters)",
                                "useful_achieved": round(useful_gbs, 1),
                                "useful_frac": round(useful_gbs / peak_gbs, 4),
                                "useful_formula": "AR bytes of the committed tokens",
                                "ar_frac": round(ar_gbs / peak_gbs, 4)},
            "greedy_equal_ar": greedy_equal_ar,
            "e2e": {"value": round(e2e, 2), "unit": UNIT,
                    "h2d_bytes_per_step": int(h2d / args.steps),
                    "d2h_bytes_per_step": int(d2h / args.steps),
                    "note": "new tokens / wall time of generate_loopspec incl. prefill"},
            "gpu_launches": None,
            "clocks": clk,
        }
        line["gpu_launches"] = int(agg["decode_kernel_launches"])
        line["gpu_launches_note"] = ("engine kernels launched by the timed decode loops "
                                     "(counted per graph replay by the engine)")
        if synth is not None:
            line["synthetic_acceptance"] = synth
        if tp_info is not None:
            line["tensor_parallel"] = tp_info
        if decode_gbs > peak_gbs:
            # more bytes per second than the measured copy peak: the byte
            # count, not the engine, is wrong
            line["decode_roofline"]["error"] = "achieved above the measured HBM peak"
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(cfg, sch, args, os.cpu_count() or 1)
        print(json.dumps(line), flush=True)
    # under tensor parallelism a peer's last kernels may still read this
    # rank's exchange region: release the engine only after every rank is done
    barrier()
    eng.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def batch_arm(args):
    """--batch B: B requests per step, split over the ranks (request i on rank
    i % N); each rank serves its share together (generate_loopspec_batch),
    with the autoregressive batch of the same prompts timed beside it."""
    from loopspec_b200.engine import Engine
    from loopspec_b200.executor import generate_loopspec_batch
    from loopspec_b200.weights import init_random_weights

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))

    def reduce(x, op):
        if dist is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=op)
        return float(t.item())

    cfg = get_config(args.config)
    sch = schedule_for(cfg, args)
    mine = list(range(rank, args.batch, world))
    lo = args.prompt_min or args.prompt

    def batch_of(step):
        g = torch.Generator().manual_seed(5000 + step)
        lens = torch.randint(lo, args.prompt + 1, (args.batch,), generator=g).tolist()
        return [make_prompt(cfg, lens[i], 100000 * step + i) for i in mine], [lens[i] for i in mine]

    weights = init_random_weights(cfg, 0, device=f"cuda:{local}", dtype=torch.bfloat16)
    eng = Engine(cfg, sch, weights, device=local, max_context=args.prompt + args.new_tokens + 64,
                 max_prompt=args.prompt, max_requests=max(1, len(mine)))
    samp = sampling_of(args)
    if args.mixed and samp is not None:
        samp = [None if i % 2 == 0 else samp for i in mine]

    def run(step, mode):
        prompts, _ = batch_of(step)
        seeds = [args.seed + 1000 * step + i for i in mine]
        t0 = time.perf_counter()
        ids, per, tot = generate_loopspec_batch(eng, prompts, args.new_tokens, sampling=samp, seeds=seeds,
                                                mode=mode)
        return ids, tot, time.perf_counter() - t0, prompts

    for i in range(args.warmup):
        run(i, "loopspec")
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = Clocks(local)
    clocks.start()
    dec_tok = dec_ms = wall = 0.0
    agg = None
    useful = 0
    for i in range(args.steps):
        ids, tot, dt, prompts = run(args.warmup + i, "loopspec")
        wall += dt
        dec_tok += tot["decode_tokens"]
        dec_ms += tot["decode_device_ms"]
        useful += roofline.useful_bytes_batch(cfg, [len(x) - 1 for x in ids], [len(p) for p in prompts])
        agg = tot if agg is None else {k: agg[k] + tot[k] for k in tot}
    torch.cuda.synchronize()
    clk = clocks.stop()
    ar_ids, ar_tot, _, _ = run(args.warmup, "ar")
    ls_ids, _, _, _ = run(args.warmup, "loopspec")
    dec_s_max = reduce(dec_ms / 1e3, dist.ReduceOp.MAX if dist else None)
    wall_max = reduce(wall, dist.ReduceOp.MAX if dist else None)
    tok_all = reduce(dec_tok, dist.ReduceOp.SUM if dist else None)
    new_all = reduce(float(sum(len(x) for x in ls_ids)) * args.steps, dist.ReduceOp.SUM if dist else None)
    ar_rate = reduce(ar_tot["decode_tokens"] / (ar_tot["decode_device_ms"] / 1e3),
                     dist.ReduceOp.SUM if dist else None)
    value = tok_all / dec_s_max
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
        peak_gbs, peak_src = float(peaks["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        peak_gbs, peak_src = 6650.0, "fallback"
    decode_gbs = roofline.decode_bytes(cfg, agg) / (dec_ms / 1e3) / 1e9
    useful_gbs = useful / (dec_ms / 1e3) / 1e9
    tp_info = tp_block(args, rank, world, local, dist) if dist is not None and not tp else None

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(1e3 * wall_max / args.steps, 1), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (uniform-random prompt ids and lengths, random-init weights seed 0)",
            "config": {"workload": f"{cfg.name} LoopSpec first={args.first} second={args.second} "
                                   f"{decode_mode(args)}{' (every other request greedy)' if args.mixed else ''}, "
                                   f"batch {args.batch} (split over {world} GPUs), "
                                   f"prompts {lo}-{args.prompt}, {args.new_tokens} new tokens",
                       "global_batch": args.batch, "seq_len": args.prompt + args.new_tokens,
                       "parallelism": f"requests split over {world} GPUs", "l2": l2_note(cfg)},
            "loopspec_tok_s": round(value, 2), "ar_tok_s": round(ar_rate, 2),
            "speedup_vs_ar": round(value / ar_rate, 3),
            "mean_accept_len": round(accept_length(agg, sch), 4),
            "counters": {k: int(agg[k]) for k in ("pipeline_cycles", "recurrent_rows", "post_rows",
                                                  "verified_proposals", "first_rejections",
                                                  "second_acceptances", "decode_tokens", "core_calls",
                                                  "core_kv_positions", "post_calls")},
            "decode_roofline": {"achieved": round(decode_gbs, 1), "peak": peak_gbs, "unit": "GB/s",
                                "frac": round(decode_gbs / peak_gbs, 4), "peak_source": peak_src,
                                "useful_frac": round(useful_gbs / peak_gbs, 4),
                                "useful_formula": "batched AR bytes of the committed tokens (weights "
                                                  "once per step for all requests, K/V per request)",
                                "rank": 0},
            "e2e": {"value": round(new_all / wall_max, 2), "unit": UNIT,
                    "note": "new tokens / wall time of the batched calls incl. prefill"},
            "greedy_equal_ar": (ls_ids == ar_ids) if samp is None else None,
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    eng.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def main():
    args = parse()
    if args.impl == "reference":
        reference_arm(args)
    else:
        from loopspec_b200.build import build
        build()
        if args.batch > 0:
            batch_arm(args)
        else:
            engine_arm(args)


if __name__ == "__main__":
    main()
