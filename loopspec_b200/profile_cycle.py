"""Profiling driver: prefill one prompt, then replay one graphed role call.

    python -m loopspec_b200.profile_cycle --config ouro-1.4b --prompt 600 \
        --lanes 4 --role core --iters 3

Runs the engine exactly as a decode cycle does (same kernels, same graph) on a
prefilled request. The replays (one warm-up, then `--iters` timed) run inside
the NVTX push/pop range "decode_replays", so an ncu launch list restricted to
it (`ncu --nvtx --nvtx-include "decode_replays/" ...`) holds exactly
(iters + 1) x kernels_per_call decode launches and none of the prefill's.
Prints the CUDA-event time per call and the number of kernels per call.
"""

from __future__ import annotations

import argparse
import json

import torch

from .build import build
from .config import get_config
from .engine import Engine
from .schedule import PipelineSchedule
from .weights import init_random_weights


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--config", default="ouro-1.4b")
    p.add_argument("--prompt", type=int, default=600)
    p.add_argument("--lanes", type=int, default=4)
    p.add_argument("--role", default="core", choices=["pre", "core", "post"])
    p.add_argument("--iters", type=int, default=3)
    p.add_argument("--first", type=int, default=1)
    p.add_argument("--second", type=int, default=2)
    p.add_argument("--sampling", action="store_true",
                   help="post role: top-p 0.9 sampling decisions instead of greedy argmax")
    p.add_argument("--decode", type=int, default=0,
                   help="> 0: after a warm-up request, decode this many greedy LoopSpec tokens inside the "
                        "NVTX range 'decode' (the device-resident loop when the schedule fits)")
    p.add_argument("--host-loop", action="store_true",
                   help="with --decode: run the cycles from the host instead of the device-resident loop")
    p.add_argument("--prefill-only", action="store_true",
                   help="time the prefill of a --prompt-token prompt (warm-up run, then one run "
                        "inside the NVTX range 'prefill') instead of a decode role call")
    a = p.parse_args()
    build()
    cfg = get_config(a.config)
    w = init_random_weights(cfg, 0, device="cuda:0", dtype=torch.bfloat16)
    X = a.second // a.first if a.second else None
    eng = Engine(cfg, PipelineSchedule(cfg.stages, a.first, X), w, device=0,
                 max_context=max(2048, a.prompt + 64), max_prompt=a.prompt, device_loop=not a.host_loop)
    g = torch.Generator().manual_seed(0)
    prompt = torch.randint(0, cfg.vocab, (a.prompt,), generator=g).tolist()
    if a.prefill_only:
        eng.generate(prompt, 1)                      # warm-up
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_push("prefill")
        _, st = eng.generate(prompt, 1)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
        print(json.dumps({"config": cfg.name, "prompt": a.prompt,
                          "prefill_device_ms": round(st["prefill_device_ms"], 3)}))
        eng.close()
        return
    if a.decode:
        eng.generate(prompt, a.decode)                  # warm-up (captures the graphs)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_push("decode")
        _, st = eng.generate(prompt, a.decode)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
        print(json.dumps({"config": cfg.name, "prompt": a.prompt, "tokens": a.decode,
                          "decode_device_ms": round(st["decode_device_ms"], 3),
                          "cycles": st["pipeline_cycles"], "host_syncs": st["host_syncs"],
                          "kernel_launches": st["decode_kernel_launches"]}))
        eng.close()
        return
    eng.prefill(prompt)
    if a.sampling:
        eng.set_sampling(1.0, 0, 0.9, 1234)
    per_call = eng.kernel_count(a.role, a.lanes)
    torch.cuda.nvtx.range_push("decode_replays")
    ms = eng.time_role(a.role, a.lanes, a.prompt, a.iters)
    torch.cuda.nvtx.range_pop()
    print(json.dumps({"config": cfg.name,
                      "role": a.role, "lanes": a.lanes, "context": a.prompt,
                      "ms_per_call": round(ms, 4), "kernels_per_call": per_call,
                      "timed_replays": a.iters, "warmup_replays": 1,
                      "launches_in_range": (a.iters + 1) * per_call}))
    eng.close()


if __name__ == "__main__":
    main()
