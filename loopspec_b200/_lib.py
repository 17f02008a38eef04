"""ctypes binding of libloopspec_engine.so (declared in include/loopspec_engine.h).

The library is built in-tree (loopspec_b200/libloopspec_engine.so) by
`loopspec_b200.build.build()`. There is no fallback: if the library is missing
or fails to load, `lib()` raises, and every engine entry point fails loudly.
"""

from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libloopspec_engine.so")

LS_OK, LS_EINVAL, LS_ECAPACITY, LS_ECUDA, LS_EDEVICE, LS_EPIPELINE = 0, -1, -2, -3, -4, -5

FAMILY = {"ouro": 0, "raven": 1}
LAYOUT = {"ouro": 0, "raven_pre": 1, "olmo_post": 2}

_i32, _i64, _f32, _f64, _u64 = (ctypes.c_int32, ctypes.c_int64, ctypes.c_float,
                                ctypes.c_double, ctypes.c_uint64)


class ModelCfg(ctypes.Structure):
    _fields_ = [
        ("family", _i32), ("layout", _i32),
        ("hidden", _i32), ("n_heads", _i32), ("n_kv_heads", _i32), ("head_dim", _i32),
        ("intermediate", _i32), ("vocab", _i32),
        ("n_pre_layers", _i32), ("n_core_layers", _i32), ("n_post_layers", _i32),
        ("stages", _i32),
        ("rope_theta", _f32), ("rms_eps", _f32), ("embed_scale", _f32), ("init_std", _f32),
        ("init_seed", _u64),
        ("qk_norm", _i32), ("adapter_bias", _i32), ("tie_embeddings", _i32),
    ]


class SchedCfg(ctypes.Structure):
    _fields_ = [
        ("step_size", _i32), ("second_step", _i32),
        ("max_context", _i32), ("max_prompt", _i32),
        ("kv_slots", _i32), ("request_rows", _i32),
        ("use_graphs", _i32), ("use_pdl", _i32), ("max_requests", _i32), ("device_loop", _i32),
    ]


class Stats(ctypes.Structure):
    _fields_ = [
        ("pipeline_cycles", _i64), ("pre_rows", _i64), ("recurrent_rows", _i64),
        ("post_rows", _i64), ("verified_proposals", _i64), ("first_rejections", _i64),
        ("second_verifications", _i64), ("second_acceptances", _i64),
        ("second_rejections", _i64), ("decode_tokens", _i64),
        ("decode_device_ms", _f64), ("decode_host_s", _f64), ("prefill_device_ms", _f64),
        ("h2d_bytes", _i64), ("d2h_bytes", _i64), ("decode_kernel_launches", _i64),
        ("pre_calls", _i64), ("core_calls", _i64), ("core_kv_positions", _i64), ("post_calls", _i64), ("host_syncs", _i64),
    ]

    def as_dict(self):
        return {name: getattr(self, name) for name, _ in self._fields_}


DECIDE_FN = ctypes.CFUNCTYPE(ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int32)
CYCLE_FN = ctypes.CFUNCTYPE(None, ctypes.c_void_p, ctypes.POINTER(ctypes.c_int64), ctypes.c_int32)
COMMIT_FN = ctypes.CFUNCTYPE(ctypes.c_int32, ctypes.c_void_p, ctypes.POINTER(ctypes.c_int64), ctypes.c_int32)
RETAIN_FN = ctypes.CFUNCTYPE(None, ctypes.c_void_p, ctypes.POINTER(ctypes.c_int64), ctypes.c_int32,
                             ctypes.c_int32)

_P = ctypes.c_void_p
TP_HANDLE_BYTES = 128   # LS_TP_HANDLE_BYTES
_PI64 = ctypes.POINTER(_i64)
_PF32 = ctypes.POINTER(_f32)

# (name, restype, argtypes) for every symbol of include/loopspec_engine.h
SIGNATURES = [
    ("ls_create", _i32, [ctypes.POINTER(ModelCfg), ctypes.POINTER(SchedCfg), _i32, ctypes.POINTER(_P)]),
    ("ls_load_weight", _i32, [_P, ctypes.c_char_p, _P, _i32, _PI64, _i32]),
    ("ls_finalize", _i32, [_P]),
    ("ls_tp_init", _i32, [_P, _i32, _i32, _P]),
    ("ls_tp_attach", _i32, [_P, _P]),
    ("ls_debug_tp_silent_peer", _i32, [_P, _i32]),
    ("ls_prefill", _i32, [_P, _PI64, _i32, _PF32, _PI64]),
    ("ls_set_sampling", _i32, [_P, _f32, _i32, _f32, _u64]),
    ("ls_cycle", _i32, [_P, _PI64, _i32, _PI64, _PF32]),
    ("ls_retain", _i32, [_P, _PI64, _PI64, _i32]),
    ("ls_generate", _i32, [_P, _PI64, _i32, _i32, _i32, _i64, _PI64, ctypes.POINTER(_i32),
                           ctypes.POINTER(Stats)]),
    ("ls_generate_stream", _i32, [_P, _PI64, _i32, _i32, _i32, _i64, COMMIT_FN, _P, _PI64,
                                  ctypes.POINTER(_i32), ctypes.POINTER(Stats)]),
    ("ls_generate_batch", _i32, [_P, _PI64, ctypes.POINTER(_i32), _i32, _i32, _i32, _i64,
                                 ctypes.POINTER(_u64), _PI64, ctypes.POINTER(_i32),
                                 ctypes.POINTER(Stats), ctypes.POINTER(Stats)]),
    ("ls_generate_batch_sampling", _i32, [_P, _PI64, ctypes.POINTER(_i32), _i32, _i32, _i32, _i64,
                                          ctypes.POINTER(_u64), ctypes.POINTER(ctypes.c_float),
                                          ctypes.POINTER(_i32), ctypes.POINTER(ctypes.c_float), _PI64,
                                          ctypes.POINTER(_i32), ctypes.POINTER(Stats),
                                          ctypes.POINTER(Stats)]),
    ("ls_device_loop_simulate", _i32, [_i32, _i32, _i32, _i64, _i32, _i64, DECIDE_FN, CYCLE_FN,
                                       RETAIN_FN, _P, _PI64, ctypes.POINTER(_i32),
                                       ctypes.POINTER(Stats)]),
    ("ls_pipeline_simulate", _i32, [_i32, _i32, _i32, _i64, _i32, _i64, DECIDE_FN, CYCLE_FN,
                                    RETAIN_FN, _P, _PI64, ctypes.POINTER(_i32),
                                    ctypes.POINTER(Stats)]),
    ("ls_time_role", _i32, [_P, _i32, _i32, _i32, _i32, ctypes.POINTER(_f64)]),
    ("ls_time_gemm", _i32, [_P, _i32, _i32, _i32, ctypes.POINTER(_f64)]),
    ("ls_time_core_gemms", _i32, [_P, _i32, _i32, ctypes.POINTER(_f64), ctypes.POINTER(_f64)]),
    ("ls_role_kernel_count", _i32, [_P, _i32, _i32, ctypes.POINTER(_i32)]),
    ("ls_debug_gemm", _i32, [_P, _i32, _i32, _PF32, _PF32]),
    ("ls_gemm_splits", _i32, [_P, _i32, ctypes.POINTER(_i32), ctypes.POINTER(_i32), ctypes.POINTER(_i32)]),
    ("ls_debug_kv", _i32, [_P, ctypes.POINTER(_P), ctypes.POINTER(_P), ctypes.POINTER(_i32),
                           ctypes.POINTER(_i32)]),
    ("ls_decode_attention_workspace_bytes", ctypes.c_size_t, [_i32, _i32, _i32, _i32, _i32]),
    ("ls_decode_attention", _i32, [_P, _P, _P, _P, _P, _P, _i32, _i32, _i32, _i32, _i32, _i32,
                                   _i32, _P, ctypes.c_size_t, _P, _P]),
    ("ls_decode_attention_noalloc", _i32, [_P, _P, _P, _P, _P, _P, _i32, _i32, _i32, _i32, _i32,
                                           _i32, _i32, _P, _P]),
    ("ls_decode_attention_noalloc_limit", ctypes.c_size_t, []),
    ("ls_destroy", _i32, [_P]),
    ("ls_last_error", ctypes.c_char_p, [_P]),
    ("ls_version", ctypes.c_char_p, []),
]

_LIB = None


def lib():
    """Load the engine library once; raise if it is missing (no CPU fallback)."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python -c 'import loopspec_b200.build as b; b.build()'`")
        handle = ctypes.CDLL(LIB_PATH)
        for name, res, args in SIGNATURES:
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = handle
    return _LIB


class EngineError(RuntimeError):
    def __init__(self, code, message):
        super().__init__(f"[{code}] {message}")
        self.code = code


def check(code, handle=None):
    if code != LS_OK:
        raise EngineError(code, lib().ls_last_error(handle).decode())
