"""Python handle over the C-ABI engine (no torch types cross the boundary).

`Engine` owns one libloopspec_engine.so handle, keeps the caller's weight
tensors alive (the engine borrows their device pointers), and converts
between Python lists / numpy arrays and the plain int64 / float buffers of
include/loopspec_engine.h.
"""

from __future__ import annotations

import ctypes

import numpy as np

from . import _lib
from .config import ModelConfig
from .schedule import PipelineSchedule


def _i64p(a):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_int64))


def _f32p(a):
    return None if a is None else a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


class Engine:
    """One looped model on one GPU: one request at a time (`generate`), or up
    to `max_requests` together (`generate_batch`)."""

    def __init__(self, cfg: ModelConfig, schedule: PipelineSchedule, weights: dict, *,
                 device: int = 0, max_context: int = 4096, max_prompt: int | None = None,
                 kv_slots: int = 0, request_rows: int = 0, use_graphs: bool = True,
                 use_pdl: bool = True, max_requests: int = 1, device_loop: bool = True):
        if schedule.stages != cfg.stages:
            raise ValueError("schedule stages must equal the model's recurrence count")
        self.cfg = cfg
        self.schedule = schedule
        self.L = _lib.lib()
        mc = _lib.ModelCfg(
            family=_lib.FAMILY[cfg.family], layout=_lib.LAYOUT[cfg.layout],
            hidden=cfg.hidden, n_heads=cfg.n_heads, n_kv_heads=cfg.n_kv_heads,
            head_dim=cfg.head_dim, intermediate=cfg.intermediate, vocab=cfg.vocab,
            n_pre_layers=cfg.n_pre_layers, n_core_layers=cfg.n_core_layers,
            n_post_layers=cfg.n_post_layers, stages=cfg.stages, rope_theta=cfg.rope_theta,
            rms_eps=cfg.rms_eps, embed_scale=cfg.embed_scale, init_std=cfg.init_std,
            init_seed=cfg.init_seed, qk_norm=int(cfg.qk_norm),
            adapter_bias=int(cfg.adapter_bias), tie_embeddings=int(cfg.tie_embeddings))
        sc = _lib.SchedCfg(
            step_size=schedule.step_size, second_step=schedule.second_step or 0,
            max_context=max_context, max_prompt=max_prompt or max_context // 2,
            kv_slots=kv_slots, request_rows=request_rows, use_graphs=int(use_graphs),
            use_pdl=int(use_pdl), max_requests=int(max_requests), device_loop=int(device_loop))
        handle = ctypes.c_void_p()
        code = self.L.ls_create(ctypes.byref(mc), ctypes.byref(sc), device, ctypes.byref(handle))
        if code != _lib.LS_OK:
            raise _lib.EngineError(code, "ls_create rejected the configuration")
        self.h = handle
        self._weights = {}
        try:
            for name, t in weights.items():
                self._load(name, t)
            _lib.check(self.L.ls_finalize(self.h), self.h)
        except Exception:
            self.close()
            raise
        self.prefill_len = None
        self.sampling = False

    def _load(self, name, t):
        import torch
        if t.dtype != torch.bfloat16 or not t.is_cuda or not t.is_contiguous():
            raise ValueError(f"{name}: weights must be contiguous bf16 CUDA tensors")
        self._weights[name] = t
        shape = np.asarray(t.shape, dtype=np.int64)
        _lib.check(self.L.ls_load_weight(self.h, name.encode(), ctypes.c_void_p(t.data_ptr()), 0,
                                         _i64p(shape), len(shape)), self.h)

    # ------------------------------------------------------ tensor parallel
    def tp_init(self, rank: int, ranks: int) -> bytes:
        """Allocate this rank's exchange region; returns the bytes every peer
        needs to map it (ls_tp_init)."""
        buf = ctypes.create_string_buffer(_lib.TP_HANDLE_BYTES)
        _lib.check(self.L.ls_tp_init(self.h, int(rank), int(ranks), buf), self.h)
        return buf.raw

    def tp_attach(self, handles) -> None:
        """Map every rank's region (ls_tp_attach); `handles` in rank order."""
        blob = b"".join(handles)
        if any(len(h) != _lib.TP_HANDLE_BYTES for h in handles):
            raise ValueError("each handle must be LS_TP_HANDLE_BYTES long")
        buf = ctypes.create_string_buffer(blob, len(blob))
        _lib.check(self.L.ls_tp_attach(self.h, buf), self.h)

    # ----------------------------------------------------------------- calls
    def prefill(self, prompt_ids, want_logits=False):
        p = np.ascontiguousarray(prompt_ids, dtype=np.int64)
        first = np.zeros(1, dtype=np.int64)
        logits = np.zeros(self.cfg.vocab, dtype=np.float32) if want_logits else None
        _lib.check(self.L.ls_prefill(self.h, _i64p(p), len(p), _f32p(logits), _i64p(first)), self.h)
        self.prefill_len = len(p) - 1
        return (int(first[0]), logits) if want_logits else int(first[0])

    def set_sampling(self, temperature=0.0, top_k=0, top_p=1.0, seed=0):
        """Request sampling settings; greedy iff top_k == 1 or temperature == 0."""
        _lib.check(self.L.ls_set_sampling(self.h, float(temperature), int(top_k), float(top_p),
                                          int(seed) & 0xFFFFFFFFFFFFFFFF), self.h)
        self.sampling = not (temperature == 0 or top_k == 1)

    def cycle(self, lanes, want_logits=False):
        """lanes: int array [n, 8] (stage, index, token, branch, parent|-1, state,
        q1 token|-1, q2 token|-1). Returns decisions int64 [n, 5]."""
        a = np.ascontiguousarray(lanes, dtype=np.int64).reshape(-1, 8)
        dec = np.zeros((len(a), 5), dtype=np.int64)
        logits = np.zeros((len(a), self.cfg.vocab), dtype=np.float32) if want_logits else None
        _lib.check(self.L.ls_cycle(self.h, _i64p(a), len(a), _i64p(dec), _f32p(logits)), self.h)
        return (dec, logits) if want_logits else dec

    def retain(self, pairs):
        b = np.ascontiguousarray([p[0] for p in pairs], dtype=np.int64)
        p = np.ascontiguousarray([-1 if p[1] is None else p[1] for p in pairs], dtype=np.int64)
        _lib.check(self.L.ls_retain(self.h, _i64p(b), _i64p(p), len(b)), self.h)

    def generate(self, prompt_ids, max_new_tokens, *, mode="loopspec", stop_token=None,
                 should_stop=None):
        """One request natively (ls_generate). should_stop(ids) -> bool, if
        given, sees the whole committed output after every commit and ends the
        request when it returns True (ls_generate_stream)."""
        p = np.ascontiguousarray(prompt_ids, dtype=np.int64)
        out = np.zeros(max_new_tokens, dtype=np.int64)
        n = ctypes.c_int32()
        st = _lib.Stats()
        m = 0 if mode == "loopspec" else 1
        stop = -1 if stop_token is None else int(stop_token)
        if should_stop is None:
            code = self.L.ls_generate(self.h, _i64p(p), len(p), max_new_tokens, m, stop, _i64p(out),
                                      ctypes.byref(n), ctypes.byref(st))
        else:
            failure = []

            def on_commit(_user, ids, k):
                try:
                    return 1 if should_stop([ids[i] for i in range(k)]) else 0
                except BaseException as ex:   # end the request, re-raise after it returns
                    failure.append(ex)
                    return 1
            cb = _lib.COMMIT_FN(on_commit)
            code = self.L.ls_generate_stream(self.h, _i64p(p), len(p), max_new_tokens, m, stop, cb, None,
                                             _i64p(out), ctypes.byref(n), ctypes.byref(st))
            if failure:
                self.prefill_len = None
                raise failure[0]
        _lib.check(code, self.h)
        self.prefill_len = None
        return out[: n.value].tolist(), st.as_dict()

    def generate_batch(self, prompts, max_new_tokens, *, mode="loopspec", stop_token=None, seeds=None,
                       sampling=None):
        """Several requests decoded together (ls_generate_batch): every cycle
        runs over the lanes of all running requests. Returns (list of ids per
        request, list of per-request stats, batch stats). Request i commits
        what it commits alone with seed seeds[i]. `sampling`, if given, is one
        entry per request: None (greedy) or {temperature, top_k, top_p}
        (ls_generate_batch_sampling; seeds are then required); otherwise every
        request uses the engine's set_sampling state."""
        lens = np.ascontiguousarray([len(p) for p in prompts], dtype=np.int32)
        flat = np.ascontiguousarray([t for p in prompts for t in p], dtype=np.int64)
        n = len(prompts)
        out = np.zeros((n, max_new_tokens), dtype=np.int64)
        n_out = np.zeros(n, dtype=np.int32)
        per = (_lib.Stats * n)()
        total = _lib.Stats()
        sd = None
        if seeds is not None:
            sd = np.ascontiguousarray([int(x) & 0xFFFFFFFFFFFFFFFF for x in seeds], dtype=np.uint64)
        m = 0 if mode == "loopspec" else 1
        stop = -1 if stop_token is None else int(stop_token)
        if sampling is not None:
            if sd is None or len(sampling) != n:
                raise ValueError("per-request sampling needs one entry and one seed per request")
            f32 = ctypes.POINTER(ctypes.c_float)
            temp = np.ascontiguousarray([0.0 if s is None else float(s.get("temperature", 1.0))
                                         for s in sampling], dtype=np.float32)
            topk = np.ascontiguousarray([1 if s is None else int(s.get("top_k", 0)) for s in sampling],
                                        dtype=np.int32)
            topp = np.ascontiguousarray([1.0 if s is None else float(s.get("top_p", 1.0))
                                         for s in sampling], dtype=np.float32)
            code = self.L.ls_generate_batch_sampling(
                self.h, _i64p(flat), lens.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), n, max_new_tokens,
                m, stop, sd.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64)), temp.ctypes.data_as(f32),
                topk.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), topp.ctypes.data_as(f32), _i64p(out),
                n_out.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), per, ctypes.byref(total))
            _lib.check(code, self.h)
            self.prefill_len = None
            return ([out[i, : n_out[i]].tolist() for i in range(n)], [per[i].as_dict() for i in range(n)],
                    total.as_dict())
        code = self.L.ls_generate_batch(
            self.h, _i64p(flat), lens.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), n, max_new_tokens, m,
            stop, None if sd is None else sd.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64)), _i64p(out),
            n_out.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), per, ctypes.byref(total))
        _lib.check(code, self.h)
        self.prefill_len = None
        ids = [out[i, : n_out[i]].tolist() for i in range(n)]
        return ids, [per[i].as_dict() for i in range(n)], total.as_dict()

    def time_role(self, role, n_lanes, context_len, iters=20):
        ms = ctypes.c_double()
        r = {"pre": 0, "core": 1, "post": 2}[role]
        _lib.check(self.L.ls_time_role(self.h, r, n_lanes, context_len, iters, ctypes.byref(ms)), self.h)
        return ms.value

    def time_gemm(self, which, n_lanes, iters=50):
        ms = ctypes.c_double()
        w = {"qkv": 0, "o": 1, "gate_up": 2, "down": 3, "lm_head": 4}[which]
        _lib.check(self.L.ls_time_gemm(self.h, w, n_lanes, iters, ctypes.byref(ms)), self.h)
        return ms.value

    def time_core_gemms(self, n_lanes, iters=5):
        """(average ms per GEMM launch, algorithmic bytes per launch) over a core-weight sweep."""
        ms, by = ctypes.c_double(), ctypes.c_double()
        _lib.check(self.L.ls_time_core_gemms(self.h, n_lanes, iters, ctypes.byref(ms),
                                             ctypes.byref(by)), self.h)
        return ms.value, by.value

    def kernel_count(self, role, n_lanes):
        c = ctypes.c_int32()
        r = {"pre": 0, "core": 1, "post": 2}[role]
        _lib.check(self.L.ls_role_kernel_count(self.h, r, n_lanes, ctypes.byref(c)), self.h)
        return c.value

    GEMMS = {"qkv": 0, "o": 1, "gate_up": 2, "down": 3, "lm_head": 4, "adapter": 5}

    def debug_gemm(self, which, x):
        """x: float32 numpy [n, K] -> float32 [n, rows] (core layer 0 weights)."""
        w = self.GEMMS[which]
        splits, rows, k = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int32()
        _lib.check(self.L.ls_gemm_splits(self.h, w, ctypes.byref(splits), ctypes.byref(rows),
                                         ctypes.byref(k)), self.h)
        x = np.ascontiguousarray(x, dtype=np.float32)
        assert x.shape[1] == k.value
        out = np.zeros((x.shape[0], rows.value), dtype=np.float32)
        _lib.check(self.L.ls_debug_gemm(self.h, w, x.shape[0], _f32p(x), _f32p(out)), self.h)
        return out, splits.value

    def close(self):
        if getattr(self, "h", None):
            self.L.ls_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
