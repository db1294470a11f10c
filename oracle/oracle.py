"""TEST INFRASTRUCTURE ONLY — the checker, never the product.

ctypes loaders for the two CPU checkers built by oracle/Makefile:

* ``Oracle`` wraps ``liboracle.so``, the C restatement of the reference sampler with the engine's
  extensions (sampler_oracle.c; lowest-index ties, presence/frequency, allow-mask, bf16).
* ``RefSampler`` wraps ``_ref/libref_sampler.so``, the reference's own ``sample()``, ``candidates()``,
  ``pick()``, ``uniform()`` and ``haru::candidates()`` compiled unmodified from its sources
  (src/families/qwen3-tts/sampler.cpp:69-116, src/common/sampling.cpp:5-19,
  src/families/haru/sampler.cpp:18-61).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU legs import this module.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libref_sampler.so")

F32, BF16 = 0, 1
MASK_NONE, MASK_BAN, MASK_ALLOW = 0, 1, 2
STATUS_NAMES = {0: "OK", 1: "PENALTY_OVERFLOW", 2: "TEMPERATURE_OVERFLOW", 3: "NO_FINITE_LOGIT",
                4: "NON_FINITE_INPUT", 5: "OTHER", 6: "INVALID"}


class Params(ctypes.Structure):
    """ssb_params / oracle_params: the reference's SamplingParams (qwen3-tts/sampler.h:12-24) + extensions."""
    _fields_ = [("greedy", ctypes.c_int32), ("temperature", ctypes.c_float), ("top_k", ctypes.c_int32),
                ("top_p", ctypes.c_float), ("repetition_penalty", ctypes.c_float),
                ("presence_penalty", ctypes.c_float), ("frequency_penalty", ctypes.c_float),
                ("flavor", ctypes.c_int32)]


def params(greedy=False, temperature=1.0, top_k=0, top_p=1.0, repetition_penalty=1.0,
           presence_penalty=0.0, frequency_penalty=0.0) -> Params:
    return Params(int(bool(greedy)), temperature, int(top_k), top_p, repetition_penalty,
                  presence_penalty, frequency_penalty, 0)


# The reference's source tree (speech.cpp), read only to compile its sampler into _ref/; the
# SPEECH_REFERENCE environment variable overrides the default location.
REFERENCE = os.environ.get("SPEECH_REFERENCE", "/root/reference")


def build(ref: bool = True) -> None:
    """Builds liboracle.so (and the reference library when its sources are present)."""
    targets = ["oracle"]
    if ref and os.path.isdir(os.path.join(REFERENCE, "src")):
        targets.append("ref")
    subprocess.run(["make", "-s", "-C", HERE, f"REF={REFERENCE}"] + targets, check=True)


def _p(a, t):
    return None if a is None else a.ctypes.data_as(ctypes.POINTER(t))


def _ptr(a):
    return None if a is None else ctypes.c_void_p(a.ctypes.data)


class Oracle:
    def __init__(self, path: str = ORACLE_SO):
        if not os.path.exists(path):
            build(ref=False)
        lib = ctypes.CDLL(path)
        self.lib = lib
        lib.oracle_sample_row.restype = ctypes.c_int
        lib.oracle_sample_row.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int32, ctypes.POINTER(Params),
                                          ctypes.POINTER(ctypes.c_int32), ctypes.c_int32,
                                          ctypes.POINTER(ctypes.c_uint32), ctypes.c_int, ctypes.c_double,
                                          ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(ctypes.c_float),
                                          ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(ctypes.c_double),
                                          ctypes.c_int32, ctypes.POINTER(ctypes.c_int32)]
        lib.oracle_sample_rows.restype = None
        lib.oracle_sample_rows.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_int32,
                                           ctypes.c_int64, ctypes.POINTER(Params), ctypes.c_int32,
                                           ctypes.POINTER(ctypes.c_int32), ctypes.c_int64,
                                           ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(ctypes.c_uint32),
                                           ctypes.c_int64, ctypes.c_int, ctypes.POINTER(ctypes.c_double),
                                           ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(ctypes.c_int32),
                                           ctypes.POINTER(ctypes.c_float)]
        lib.oracle_pick.restype = ctypes.c_int32
        lib.oracle_pick.argtypes = [ctypes.POINTER(ctypes.c_double), ctypes.c_int32, ctypes.c_double]
        lib.oracle_uniform.restype = None
        lib.oracle_uniform.argtypes = [ctypes.c_uint64, ctypes.c_int64, ctypes.POINTER(ctypes.c_double)]
        _bind_dry(lib, "oracle_dry_run")
        lib.oracle_haru_shape.restype = None
        lib.oracle_haru_shape.argtypes = [ctypes.POINTER(ctypes.c_float), ctypes.POINTER(ctypes.c_int32),
                                          ctypes.POINTER(ctypes.c_double), ctypes.c_int32,
                                          ctypes.POINTER(ctypes.c_float), ctypes.c_int32, ctypes.c_int32,
                                          ctypes.c_int32, ctypes.c_float, ctypes.c_int32]
        for name in ("oracle_haru_candidates", "oracle_drama3_candidates"):
            f = getattr(lib, name)
            f.restype = ctypes.c_int
            f.argtypes = [ctypes.POINTER(ctypes.c_float), ctypes.c_int32, ctypes.c_float, ctypes.c_int32,
                          ctypes.c_float, ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(ctypes.c_double),
                          ctypes.c_int32, ctypes.POINTER(ctypes.c_int32)]

    def sample_row(self, logits, p: Params, history=None, mask=None, mask_kind=MASK_NONE, u=0.0, cap=0,
                   want_processed=False):
        """One row: returns dict(status, id, processed, tokens, weights, count)."""
        dtype = BF16 if logits.dtype == np.uint16 else F32
        logits = np.ascontiguousarray(logits)
        n = logits.shape[-1]
        h = None if history is None else np.ascontiguousarray(history, dtype=np.int32)
        m = None if mask is None else np.ascontiguousarray(mask, dtype=np.uint32)
        out_id = ctypes.c_int32(-1)
        count = ctypes.c_int32(0)
        processed = np.empty(n, np.float32) if want_processed else None
        tokens = np.empty(max(cap, 1), np.int32)
        weights = np.empty(max(cap, 1), np.float64)
        st = self.lib.oracle_sample_row(_ptr(logits), dtype, n, ctypes.byref(p), _p(h, ctypes.c_int32),
                                        0 if h is None else len(h), _p(m, ctypes.c_uint32), mask_kind, float(u),
                                        ctypes.byref(out_id), _p(processed, ctypes.c_float),
                                        _p(tokens, ctypes.c_int32), _p(weights, ctypes.c_double), cap,
                                        ctypes.byref(count))
        c = min(count.value, cap)
        return dict(status=st, id=out_id.value, processed=processed, tokens=tokens[:c].copy(),
                    weights=weights[:c].copy(), count=count.value)

    def sample_rows(self, logits, p, history=None, hlens=None, mask=None, mask_kind=MASK_NONE, u=None,
                    want_processed=False):
        """Rows of a [B, V] array (f32, or uint16 holding bf16 bits). p: Params or a list of Params."""
        logits = np.ascontiguousarray(logits)
        b, n = logits.shape
        dtype = BF16 if logits.dtype == np.uint16 else F32
        per_row = isinstance(p, (list, tuple))
        parr = (Params * b)(*p) if per_row else (Params * 1)(p)
        h = None if history is None else np.ascontiguousarray(history, dtype=np.int32)
        hl = None if hlens is None else np.ascontiguousarray(hlens, dtype=np.int32)
        m = None if mask is None else np.ascontiguousarray(mask, dtype=np.uint32)
        mask_ld = 0 if m is None or m.ndim == 1 else m.shape[1]
        uu = None if u is None else np.ascontiguousarray(u, dtype=np.float64)
        ids = np.empty(b, np.int32)
        status = np.empty(b, np.int32)
        processed = np.empty((b, n), np.float32) if want_processed else None
        self.lib.oracle_sample_rows(_ptr(logits), dtype, b, n, n, parr, int(per_row), _p(h, ctypes.c_int32),
                                    0 if h is None else h.shape[1], _p(hl, ctypes.c_int32), _p(m, ctypes.c_uint32),
                                    mask_ld, mask_kind, _p(uu, ctypes.c_double), _p(ids, ctypes.c_int32),
                                    _p(status, ctypes.c_int32), _p(processed, ctypes.c_float))
        return ids, status, processed

    def pick(self, weights, u) -> int:
        w = np.ascontiguousarray(weights, dtype=np.float64)
        return self.lib.oracle_pick(_p(w, ctypes.c_double), len(w), float(u))

    def uniform(self, seed: int, n: int):
        out = np.empty(n, np.float64)
        self.lib.oracle_uniform(seed, n, _p(out, ctypes.c_double))
        return out

    def dry_run(self, cfg, exempt, tokens, cap=256):
        """Dry::update over `tokens` (haru/sampler.cpp:86-110): penalties after each step
        (tokens [n, cap], values [n, cap], counts [n])."""
        return _dry_run(self.lib.oracle_dry_run, cfg, exempt, tokens, cap)

    def haru_shape(self, logits, pen_tokens, pen_values, silent, pad, eop, eos, eop_bias, must_speak):
        """shape_logits (haru/sampler.cpp:116-124) of one f32 row (a copy is returned)."""
        x = np.array(logits, np.float32)
        pt = np.ascontiguousarray(pen_tokens, np.int32)
        pv = np.ascontiguousarray(pen_values, np.float64)
        sil = np.ascontiguousarray(silent, np.float32)
        self.lib.oracle_haru_shape(_p(x, ctypes.c_float), _p(pt, ctypes.c_int32), _p(pv, ctypes.c_double), len(pt),
                                   _p(sil, ctypes.c_float), pad, eop, eos, eop_bias, int(must_speak))
        return x

    def _family(self, f, logits, temperature, top_k, top_p, cap):
        x = np.ascontiguousarray(logits, dtype=np.float32)
        cap = len(x) if cap is None else cap
        tokens = np.empty(max(cap, 1), np.int32)
        weights = np.empty(max(cap, 1), np.float64)
        count = ctypes.c_int32(0)
        st = f(_p(x, ctypes.c_float), len(x), temperature, top_k, top_p, _p(tokens, ctypes.c_int32),
               _p(weights, ctypes.c_double), cap, ctypes.byref(count))
        c = min(count.value, cap)
        return st, tokens[:c].copy(), weights[:c].copy()

    def haru_candidates(self, logits, temperature, top_k, top_p, cap=None):
        """haru::candidates (haru/sampler.cpp:18-61): (status, tokens, weights)."""
        return self._family(self.lib.oracle_haru_candidates, logits, temperature, top_k, top_p, cap)

    def drama3_candidates(self, logits, temperature, top_k, top_p, cap=None):
        """drama3::candidates (drama3/sampler.cpp:30-60): (status, tokens, weights)."""
        return self._family(self.lib.oracle_drama3_candidates, logits, temperature, top_k, top_p, cap)


class DryConfig(ctypes.Structure):
    """ssb_dry_config / haru::DryConfig (haru/sampler.h:37-40)."""
    _fields_ = [("multiplier", ctypes.c_double), ("base", ctypes.c_double), ("max_penalty", ctypes.c_double),
                ("allowed_length", ctypes.c_int32), ("lookback", ctypes.c_int32),
                ("max_match_length", ctypes.c_int32), ("reserved", ctypes.c_int32)]


def _dry_run(f, cfg, exempt, tokens, cap):
    ex = np.ascontiguousarray(exempt, np.int32)
    t = np.ascontiguousarray(tokens, np.int32)
    n = len(t)
    pt = np.full((n, cap), -1, np.int32)
    pv = np.zeros((n, cap))
    cnt = np.zeros(n, np.int32)
    f(ctypes.byref(cfg), _p(ex, ctypes.c_int32), len(ex), _p(t, ctypes.c_int32), n, _p(pt, ctypes.c_int32),
      _p(pv, ctypes.c_double), cap, _p(cnt, ctypes.c_int32))
    return pt, pv, cnt


def _bind_dry(lib, run_name):
    f = getattr(lib, run_name)
    f.restype = None
    f.argtypes = [ctypes.POINTER(DryConfig), ctypes.POINTER(ctypes.c_int32), ctypes.c_int32,
                  ctypes.POINTER(ctypes.c_int32), ctypes.c_int64, ctypes.POINTER(ctypes.c_int32),
                  ctypes.POINTER(ctypes.c_double), ctypes.c_int32, ctypes.POINTER(ctypes.c_int32)]


class RefSampler:
    """The reference's own sampler (compiled from its sources into oracle/_ref)."""

    def __init__(self, path: str = REF_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} is not built (oracle/Makefile ref target; needs the reference sources)")
        lib = ctypes.CDLL(path)
        self.lib = lib
        i32p, f32p, f64p, u8p = (ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(ctypes.c_float),
                                 ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_uint8))
        lib.ref_sample.restype = ctypes.c_int
        lib.ref_sample.argtypes = [f32p, ctypes.c_int32, ctypes.POINTER(Params), i32p, ctypes.c_int32, u8p,
                                   ctypes.c_int32, ctypes.c_double, i32p]
        lib.ref_candidates.restype = ctypes.c_int
        lib.ref_candidates.argtypes = [f32p, ctypes.c_int32, ctypes.POINTER(Params), i32p, ctypes.c_int32, u8p,
                                       ctypes.c_int32, i32p, f64p, ctypes.c_int32, i32p]
        lib.ref_pick.restype = ctypes.c_int32
        lib.ref_pick.argtypes = [f64p, ctypes.c_int32, ctypes.c_double]
        lib.ref_uniform.restype = None
        lib.ref_uniform.argtypes = [ctypes.c_uint64, ctypes.c_int64, f64p]
        _bind_dry(lib, "ref_dry_run")
        lib.ref_haru_shape.restype = None
        lib.ref_haru_shape.argtypes = [f32p, ctypes.c_int32, ctypes.POINTER(DryConfig), i32p, ctypes.c_int32, i32p,
                                       ctypes.c_int64, f32p, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                       ctypes.c_float, ctypes.c_int32]
        for name in ("ref_haru_candidates", "ref_drama3_candidates"):
            f = getattr(lib, name)
            f.restype = ctypes.c_int
            f.argtypes = [f32p, ctypes.c_int32, ctypes.c_float, ctypes.c_int32, ctypes.c_float, i32p, f64p,
                          ctypes.c_int32, i32p]
        lib.ref_time_rows.restype = ctypes.c_double
        lib.ref_time_rows.argtypes = [f32p, ctypes.c_int64, ctypes.c_int32, ctypes.c_int64, ctypes.POINTER(Params),
                                      i32p, ctypes.c_int64, i32p, u8p, ctypes.c_int64, f64p, ctypes.c_int32,
                                      i32p, i32p]
        lib.ref_hardware_concurrency.restype = ctypes.c_int32
        lib.ref_last_message.restype = ctypes.c_char_p

    @staticmethod
    def _banned(banned):
        return None if banned is None else np.ascontiguousarray(banned, dtype=np.uint8)

    def sample(self, logits, p: Params, history=None, banned=None, u=0.0):
        x = np.ascontiguousarray(logits, dtype=np.float32)
        h = None if history is None else np.ascontiguousarray(history, dtype=np.int32)
        b = self._banned(banned)
        out = ctypes.c_int32(-1)
        st = self.lib.ref_sample(_p(x, ctypes.c_float), len(x), ctypes.byref(p), _p(h, ctypes.c_int32),
                                 0 if h is None else len(h), _p(b, ctypes.c_uint8), 0 if b is None else len(b),
                                 float(u), ctypes.byref(out))
        return st, out.value

    def candidates(self, logits, p: Params, history=None, banned=None, cap=None):
        x = np.ascontiguousarray(logits, dtype=np.float32)
        cap = len(x) if cap is None else cap
        h = None if history is None else np.ascontiguousarray(history, dtype=np.int32)
        b = self._banned(banned)
        tokens = np.empty(cap, np.int32)
        weights = np.empty(cap, np.float64)
        count = ctypes.c_int32(0)
        st = self.lib.ref_candidates(_p(x, ctypes.c_float), len(x), ctypes.byref(p), _p(h, ctypes.c_int32),
                                     0 if h is None else len(h), _p(b, ctypes.c_uint8), 0 if b is None else len(b),
                                     _p(tokens, ctypes.c_int32), _p(weights, ctypes.c_double), cap,
                                     ctypes.byref(count))
        c = min(count.value, cap)
        return st, tokens[:c].copy(), weights[:c].copy()

    def pick(self, weights, u) -> int:
        w = np.ascontiguousarray(weights, dtype=np.float64)
        return self.lib.ref_pick(_p(w, ctypes.c_double), len(w), float(u))

    def uniform(self, seed: int, n: int):
        out = np.empty(n, np.float64)
        self.lib.ref_uniform(seed, n, _p(out, ctypes.c_double))
        return out

    def haru_candidates(self, logits, temperature, top_k, top_p, cap=None):
        return Oracle._family(self, self.lib.ref_haru_candidates, logits, temperature, top_k, top_p, cap)

    def drama3_candidates(self, logits, temperature, top_k, top_p, cap=None):
        return Oracle._family(self, self.lib.ref_drama3_candidates, logits, temperature, top_k, top_p, cap)

    def dry_run(self, cfg, exempt, tokens, cap=256):
        return _dry_run(self.lib.ref_dry_run, cfg, exempt, tokens, cap)

    def haru_shape(self, logits, cfg, exempt, tokens, silent, pad, eop, eos, eop_bias, must_speak):
        """shape_logits with the reference's own Dry after `tokens` (a copy is returned)."""
        x = np.array(logits, np.float32)
        ex = np.ascontiguousarray(exempt, np.int32)
        t = np.ascontiguousarray(tokens, np.int32)
        sil = np.ascontiguousarray(silent, np.float32)
        self.lib.ref_haru_shape(_p(x, ctypes.c_float), len(x), ctypes.byref(cfg), _p(ex, ctypes.c_int32), len(ex),
                                _p(t, ctypes.c_int32), len(t), _p(sil, ctypes.c_float), pad, eop, eos, eop_bias,
                                int(must_speak))
        return x

    def time_rows(self, logits_f32, p: Params, history=None, hlens=None, banned=None, u=None, threads=1):
        """sample() over every row with `threads` workers; returns (seconds, ids, status)."""
        x = np.ascontiguousarray(logits_f32, dtype=np.float32)
        rows, n = x.shape
        h = None if history is None else np.ascontiguousarray(history, dtype=np.int32)
        hl = None if hlens is None else np.ascontiguousarray(hlens, dtype=np.int32)
        b = self._banned(banned)
        banned_ld = 0 if b is None or b.ndim == 1 else b.shape[1]
        uu = np.zeros(rows, np.float64) if u is None else np.ascontiguousarray(u, dtype=np.float64)
        ids = np.empty(rows, np.int32)
        status = np.empty(rows, np.int32)
        secs = self.lib.ref_time_rows(_p(x, ctypes.c_float), rows, n, n, ctypes.byref(p), _p(h, ctypes.c_int32),
                                      0 if h is None else h.shape[1], _p(hl, ctypes.c_int32), _p(b, ctypes.c_uint8),
                                      banned_ld, _p(uu, ctypes.c_double), threads, _p(ids, ctypes.c_int32),
                                      _p(status, ctypes.c_int32))
        if secs < 0:
            raise ValueError("ref_time_rows refused its arguments")
        return secs, ids, status

    def hardware_concurrency(self) -> int:
        return self.lib.ref_hardware_concurrency()


def ref_available() -> bool:
    return os.path.exists(REF_SO)
