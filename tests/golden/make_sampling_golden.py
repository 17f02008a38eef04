"""Golden decision rows of the reference's own sampling code.

Runs the unmodified reference modules sglang_recurrent/loopspec/sampling/
{policy,sampler,rejection,distributions}.py and loopspec/decisions.py on the
CPU, through their public entry points SamplingDecisionPolicy.queue / read
(policy.py:220-283):

* TRITON_INTERPRET=1 makes Triton execute sampler.py's @triton.jit kernels
  with numpy instead of on a GPU.
* The CUDA guards (distributions.py:39-40 and 102-103) see logits as a tensor
  subclass whose only change is to report is_cuda == True.
* The policy, CategoricalSampler, RejectionSampler and DecisionReadback
  objects are assembled without their constructors (which demand a CUDA
  device and pinned memory), with CPU buffers of the shapes the constructors
  allocate (policy.py:22-68, sampler.py:473-506, rejection.py:99-139,
  decisions.py:54-64); CUDA events become no-ops, and the rejection graph's
  replay runs RejectionSampler._run directly (the operations the captured
  graph records).
* torch.rand is wrapped to record every uniform the policy draws, in order,
  so the oracle can replay each decision with the same uniforms.

The readout logits follow tests/golden/sampling_cases.py. Writes
sampling_golden.json beside this script. Run where the reference tree is:
    python tests/golden/make_sampling_golden.py [reference_root]
"""

from __future__ import annotations

import json
import os
import sys
import types

os.environ["TRITON_INTERPRET"] = "1"

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

import torch  # noqa: E402

from sampling_cases import KIND_NAMES, SCENARIOS, cycle_rows, readout_logits  # noqa: E402

MAX_ROWS = 8


class _Event:
    def record(self):
        pass

    def synchronize(self):
        pass


class _GraphReplay:
    """Stands in for the captured rejection graph: replays _run's operations."""

    def __init__(self, rejections):
        self.rejections = rejections

    def replay(self):
        self.rejections._run()


class _DeviceTag(torch.Tensor):
    """A CPU tensor that answers is_cuda == True (nothing else changes)."""

    @property
    def is_cuda(self):
        return True


def load_reference(root):
    sys.path.insert(0, root)
    from sglang_recurrent.loopspec import decisions
    from sglang_recurrent.loopspec.sampling import policy, rejection, sampler
    return decisions, policy, rejection, sampler


def build_policy(ref, vocab, options, generator):
    decisions, policy_mod, rejection_mod, sampler_mod = ref
    s = object.__new__(sampler_mod.CategoricalSampler)
    s.max_rows = MAX_ROWS
    s.vocabulary_size = vocab
    s.chunk_size = 2048
    s.chunks = (vocab + 2047) // 2048
    s.chunk_sums = torch.empty((MAX_ROWS, s.chunks), dtype=torch.float32)
    s.top_p_chunk_sums = torch.empty_like(s.chunk_sums)
    s.uniforms = torch.empty(MAX_ROWS, dtype=torch.float32)
    s.samples = torch.empty((3, MAX_ROWS), dtype=torch.int64)
    s.verification_decisions = torch.empty((MAX_ROWS, 5), dtype=torch.int64)
    s.proposal_actions = torch.empty(MAX_ROWS, dtype=torch.int64)
    r = object.__new__(rejection_mod.RejectionSampler)
    r.vocabulary_size = vocab
    r.device = torch.device("cpu")
    r.sample_with_uniforms = s._sample_with_uniforms
    r.first = torch.zeros((1, vocab), dtype=torch.float32)
    r.target = torch.zeros_like(r.first)
    r.second = torch.zeros_like(r.first)
    r.metadata = torch.zeros(2, dtype=torch.int64)
    r.metadata_host = torch.zeros(2, dtype=torch.int64)
    r.uniforms = torch.empty(2, dtype=torch.float32)
    r.sample = torch.empty(1, dtype=torch.int64)
    r.graph = _GraphReplay(r)
    s.rejections = r
    rb = object.__new__(decisions.DecisionReadback)
    rb.host = torch.empty(MAX_ROWS * 5, dtype=torch.int64)
    rb.ready = _Event()
    p = object.__new__(policy_mod.SamplingDecisionPolicy)
    p.readback = rb
    p.options = options
    p.sampler = s
    p.generator = generator
    p.constants = torch.tensor([0, 1], dtype=torch.int64)
    for name in ("proposal_token", "verification_token", "sample_row"):
        setattr(p, name + "_host", torch.empty(MAX_ROWS, dtype=torch.int64))
        setattr(p, name + "_device", torch.empty(MAX_ROWS, dtype=torch.int64))
    p.rejection_host = torch.empty((MAX_ROWS, 3), dtype=torch.int64)
    p.rejection_ready = _Event()
    p.top_p_thresholds = torch.full((MAX_ROWS, 1), options["top_p"], dtype=torch.float32)
    return p


def run_scenario(ref, scenario):
    name, vocab, T, top_k, top_p, has_q2, scale, noise, cycles, seed = scenario
    options = {"temperature": T, "top_k": top_k if top_k else 1 << 30, "top_p": top_p}
    gen = torch.Generator().manual_seed(seed)
    policy = build_policy(ref, vocab, options, gen)
    draws = []
    real_rand = torch.rand

    def recording_rand(*size, out=None, generator=None, **kw):
        res = real_rand(*size, out=out, generator=generator, **kw)
        draws.append([float(x) for x in res.reshape(-1).tolist()])
        return res

    lanes = {}
    out_cycles = []
    torch.rand = recording_rand
    try:
        for t in range(cycles):
            rows = cycle_rows(t, cycles, has_q2)
            if not rows:
                continue
            for n, _ in rows:
                lanes.setdefault(n, types.SimpleNamespace(first_token=None, first_state=None,
                                                          second_token=None, second_state=None))
            row_lanes = [lanes[n] for n, _ in rows]
            endpoints = {i: KIND_NAMES[k] for i, (_, k) in enumerate(rows)}
            before = [(ln.first_token, ln.second_token) for ln in row_lanes]
            logits = torch.stack([readout_logits(vocab, scale, noise, seed, n, k) for n, k in rows])
            post = types.SimpleNamespace(next_token_logits=logits.as_subclass(_DeviceTag))
            draws.clear()
            batch = policy.queue(post, endpoints, row_lanes)
            decisions = policy.read(row_lanes, endpoints, batch)
            call = {"t": t, "rows": [[n, k] for n, k in rows], "lanes_before": before,
                    "draws": list(draws), "decisions": [list(map(int, decisions[i])) for i in range(len(rows))]}
            out_cycles.append(call)
            for i, (n, k) in enumerate(rows):
                d = decisions[i]
                ln = lanes[n]
                if k == 0:
                    ln.first_token = int(d[0])
                    ln.first_state = batch.proposal_states[i].as_subclass(torch.Tensor).clone()
                elif k == 1 and d[1]:
                    ln.second_token = int(d[0])
                    ln.second_state = batch.proposal_states[i].as_subclass(torch.Tensor).clone()
    finally:
        torch.rand = real_rand
    return {"name": name, "vocab": vocab, "temperature": T, "top_k": top_k, "top_p": top_p,
            "has_q2": has_q2, "scale": scale, "noise": noise, "cycles": cycles, "seed": seed,
            "calls": out_cycles}


def main():
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("LOOPSPEC_REFERENCE", "/root/reference")
    ref = load_reference(root)
    torch.set_num_threads(1)
    out = {"source": "sglang_recurrent/loopspec/sampling/policy.py SamplingDecisionPolicy.queue/read "
                     "(reference code, Triton interpreter on CPU)",
           "scenarios": [run_scenario(ref, sc) for sc in SCENARIOS]}
    path = os.path.join(HERE, "sampling_golden.json")
    with open(path, "w") as f:
        json.dump(out, f, separators=(",", ":"))
    n = sum(len(c["decisions"]) for sc in out["scenarios"] for c in sc["calls"])
    print(f"wrote {path}: {len(out['scenarios'])} scenarios, {n} decision rows")


if __name__ == "__main__":
    main()
