"""CPU oracle for the LoopSpec decode step -- TEST INFRASTRUCTURE ONLY.

Nothing in the product package (`loopspec_b200`) imports this package. Only
`tests/`, `__graft_entry__.smoke()` and `bench.py`'s CPU-baseline leg use it,
and only as the checker or as the timed CPU reference arm.

Contents:
  pipeline.py  -- restatement of the reference scheduler
                  (sglang_recurrent/loopspec/pipeline.py) and of the greedy
                  decision rules (sglang_recurrent/loopspec/decisions.py).
  model.py     -- fp32 PyTorch CPU restatement of the model roles
                  (sglang_recurrent/modeling/{ouro,raven,components}.py).
  executor.py  -- a PipelineExecutor over model.py with per-branch,
                  per-role/depth KV timelines (loopspec/executor.py,
                  loopspec/request.py, loopspec/branching/manager.py), plus the
                  unrolled autoregressive path (modeling/serving.py:185-239).
  sampling.py  -- float64 restatement of the top-p / temperature sampler,
                  the q2 residual draft and the verification rule
                  (loopspec/sampling/{distributions,sampler,policy,rejection}.py).

Parity pins: pipeline.py is checked against traces recorded by driving the
reference's own `continue_pipelined` (tests/golden/make_pipeline_golden.py).
The model math has no golden vectors in the reference (it ships no tests);
that part is pinned by self-consistency (LoopSpec == AR) and by the
transformers Llama/OLMo2 layer cross-check where one applies.
"""
