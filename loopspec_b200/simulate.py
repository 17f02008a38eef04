"""Run the engine's native scheduler loop with host-side decisions (no GPU).

`simulate_pipeline` drives the same C++ code that `ls_generate` runs between
GPU cycles (continue_pipelined + greedy resolve + state-slot pool + counters),
with readout tokens supplied by a Python function. Used to check the native
scheduler against traces of the reference scheduler.
"""

from __future__ import annotations

import ctypes

import numpy as np

from . import _lib

KINDS = ("q1", "q2", "final")


def simulate_pipeline(stages, step_size, second_step, first_token, max_new_tokens, decide,
                      *, stop_token=None, device_logic=False):
    """decide(index, token, kind) -> int. Returns (ids, stats, trace).
    device_logic: run the device loop's scheduler (dev_sched.cuh, compiled for
    the host) instead of the host scheduler."""
    L = _lib.lib()
    trace = []
    errors = []

    def _decide(user, index, token, kind):
        try:
            return int(decide(int(index), int(token), KINDS[kind]))
        except Exception as exc:  # surface Python errors after the call
            errors.append(exc)
            return 0

    def _cycle(user, lanes, n):
        rows = [[lanes[7 * i + j] for j in range(7)] for i in range(n)]
        trace.append({"lanes": rows})

    def _retain(user, pairs, n, accepted):
        trace.append({"retain": sorted([pairs[2 * i], pairs[2 * i + 1]] for i in range(n)),
                      "accepted_stage": accepted})

    cb_d, cb_c, cb_r = _lib.DECIDE_FN(_decide), _lib.CYCLE_FN(_cycle), _lib.RETAIN_FN(_retain)
    out = np.zeros(max(max_new_tokens, 1), dtype=np.int64)
    n = ctypes.c_int32()
    st = _lib.Stats()
    fn = L.ls_device_loop_simulate if device_logic else L.ls_pipeline_simulate
    code = fn(
        stages, step_size, second_step or 0, first_token, max_new_tokens,
        -1 if stop_token is None else stop_token, cb_d, cb_c, cb_r, None,
        out.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)), ctypes.byref(n), ctypes.byref(st))
    if errors:
        raise errors[0]
    _lib.check(code)
    return out[: n.value].tolist(), st.as_dict(), trace
