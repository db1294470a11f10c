"""Python binding of libspeech_sampler_b200.so (the C ABI of include/speech_sampler_b200.h).

A thin ctypes layer: it passes raw device pointers (from torch tensors, which serve only as device
memory and streams here) or host pointers (numpy) to the CUDA engine, and raises on failure. There
is no CPU fallback: if the library is missing or no GPU is present, construction fails.

    s = Sampler(device=0)
    ids, status = s.sample(logits, params(temperature=0.9, top_k=50), history=h, u=u)

The settings mirror the reference's SamplingParams (src/families/qwen3-tts/sampler.h:12-24) plus the
presence/frequency extensions; per-row statuses mirror its refusals (ROW_* below).
"""
from __future__ import annotations

import ctypes
import os
import re

import numpy as np

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
LIB_PATH = os.path.join(PKG, "libspeech_sampler_b200.so")
HEADER = os.path.join(ROOT, "include", "speech_sampler_b200.h")

OK, INVALID_ARGUMENT, OUT_OF_RANGE, DEVICE, OUT_OF_MEMORY = range(5)
(ROW_OK, ROW_PENALTY_OVERFLOW, ROW_TEMPERATURE_OVERFLOW, ROW_NO_FINITE_LOGIT, ROW_NON_FINITE_INPUT, ROW_INVALID_ROW,
 ROW_DEVICE_TIMEOUT) = range(7)
F32, BF16 = 0, 1
MASK_NONE, MASK_BAN, MASK_ALLOW = 0, 1, 2
SMALL_VOCAB = 8192
MAX_STREAM_HISTORY = 8192
STREAM_MAX_K = 1024


class SsbError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"ssb status {status}: {message}")
        self.status = status
        self.message = message


class Params(ctypes.Structure):
    _fields_ = [("greedy", ctypes.c_int32), ("temperature", ctypes.c_float), ("top_k", ctypes.c_int32),
                ("top_p", ctypes.c_float), ("repetition_penalty", ctypes.c_float),
                ("presence_penalty", ctypes.c_float), ("frequency_penalty", ctypes.c_float),
                ("flavor", ctypes.c_int32)]


FLAVOR_QWEN3_TTS, FLAVOR_HARU, FLAVOR_DRAMA3 = 0, 1, 2


def params(greedy=False, temperature=1.0, top_k=0, top_p=1.0, repetition_penalty=1.0, presence_penalty=0.0,
           frequency_penalty=0.0, flavor=FLAVOR_QWEN3_TTS) -> Params:
    """The reference's SamplingParams defaults (qwen3-tts/sampler.h:12-24) plus the extensions; `flavor`
    selects the candidate rules of the Haru (haru/sampler.cpp:18-61) or Drama 3
    (drama3/sampler.cpp:18-59) families instead of Qwen3-TTS's."""
    return Params(int(bool(greedy)), temperature, int(top_k), top_p, repetition_penalty, presence_penalty,
                  frequency_penalty, int(flavor))


PARAMS_DTYPE = np.dtype([("greedy", "<i4"), ("temperature", "<f4"), ("top_k", "<i4"), ("top_p", "<f4"),
                         ("repetition_penalty", "<f4"), ("presence_penalty", "<f4"),
                         ("frequency_penalty", "<f4"), ("flavor", "<i4")])


def params_array(plist) -> np.ndarray:
    """A [rows] structured array of ssb_params (for row_params)."""
    a = np.zeros(len(plist), PARAMS_DTYPE)
    for i, p in enumerate(plist):
        a[i] = (p.greedy, p.temperature, p.top_k, p.top_p, p.repetition_penalty, p.presence_penalty,
                p.frequency_penalty, p.flavor)
    return a


class Rows(ctypes.Structure):
    _fields_ = [("logits", ctypes.c_void_p), ("ld", ctypes.c_int64), ("dtype", ctypes.c_int32),
                ("rows", ctypes.c_int32), ("vocab", ctypes.c_int32), ("max_top_k", ctypes.c_int32),
                ("params", Params), ("row_params", ctypes.c_void_p), ("history", ctypes.c_void_p),
                ("history_ld", ctypes.c_int64), ("history_len", ctypes.c_void_p), ("mask", ctypes.c_void_p),
                ("mask_ld", ctypes.c_int64), ("mask_kind", ctypes.c_int32), ("reserved", ctypes.c_int32),
                ("u", ctypes.c_void_p), ("ids", ctypes.c_void_p), ("status", ctypes.c_void_p)]


class DryConfig(ctypes.Structure):
    """ssb_dry_config: haru::DryConfig (haru/sampler.h:37-40)."""
    _fields_ = [("multiplier", ctypes.c_double), ("base", ctypes.c_double), ("max_penalty", ctypes.c_double),
                ("allowed_length", ctypes.c_int32), ("lookback", ctypes.c_int32),
                ("max_match_length", ctypes.c_int32), ("reserved", ctypes.c_int32)]


class HaruShape(ctypes.Structure):
    """ssb_haru_shape: shape_logits()'s inputs for rows on the device (haru/sampler.cpp:116-124)."""
    _fields_ = [("logits", ctypes.c_void_p), ("ld", ctypes.c_int64), ("rows", ctypes.c_int32),
                ("vocab", ctypes.c_int32), ("silent", ctypes.c_void_p), ("silent_ld", ctypes.c_int64),
                ("pad", ctypes.c_int32), ("eop", ctypes.c_int32), ("eos", ctypes.c_int32),
                ("eop_bias", ctypes.c_float), ("must_speak", ctypes.c_void_p)]


class Embed(ctypes.Structure):
    """ssb_embed: the table the drawn ids index (ggml_get_rows of the chain's next step)."""
    _fields_ = [("table", ctypes.c_void_p), ("ld", ctypes.c_int64), ("table_rows", ctypes.c_int32),
                ("dtype", ctypes.c_int32), ("dim", ctypes.c_int32), ("reserved", ctypes.c_int32),
                ("out", ctypes.c_void_p), ("out_ld", ctypes.c_int64)]


class LmHead(ctypes.Structure):
    """ssb_lm_head: the LM head fused with its argmax."""
    _fields_ = [("hidden", ctypes.c_void_p), ("hidden_ld", ctypes.c_int64), ("rows", ctypes.c_int32),
                ("dim", ctypes.c_int32), ("weight", ctypes.c_void_p), ("weight_ld", ctypes.c_int64),
                ("vocab", ctypes.c_int32), ("dtype", ctypes.c_int32), ("ids", ctypes.c_void_p),
                ("max_logit", ctypes.c_void_p), ("status", ctypes.c_void_p)]


def header_symbols(path: str = HEADER):
    """Every function the C header declares (SSB_API ... name(...))."""
    text = open(path).read()
    return re.findall(r"SSB_API\s+[^;(]*?\b(ssb_\w+)\s*\(", text)


_LIB = None


def load_library(path: str = LIB_PATH):
    """Loads the engine. Raises if it is not built — there is no fallback."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not os.path.exists(path):
        raise FileNotFoundError(f"{path} is not built: run python speech.cpp_b200/speech_build.py")
    lib = ctypes.CDLL(path)
    vp, i32 = ctypes.c_void_p, ctypes.c_int32
    lib.ssb_version.restype = ctypes.c_char_p
    lib.ssb_last_error.restype = ctypes.c_char_p
    lib.ssb_context_create.restype = ctypes.c_int
    lib.ssb_context_create.argtypes = [i32, ctypes.POINTER(vp)]
    lib.ssb_context_destroy.restype = ctypes.c_int
    lib.ssb_context_destroy.argtypes = [vp]
    lib.ssb_context_reserve.restype = ctypes.c_int
    lib.ssb_context_reserve.argtypes = [vp, i32, i32]
    lib.ssb_sample_rows.restype = ctypes.c_int
    lib.ssb_sample_rows.argtypes = [vp, ctypes.POINTER(Rows), vp]
    lib.ssb_candidates_rows.restype = ctypes.c_int
    lib.ssb_candidates_rows.argtypes = [vp, ctypes.POINTER(Rows), i32, vp, vp, vp, vp, vp]
    lib.ssb_sample_host.restype = ctypes.c_int
    lib.ssb_sample_host.argtypes = [vp, ctypes.POINTER(Rows), vp]
    lib.ssb_restrict_rows.restype = ctypes.c_int
    lib.ssb_restrict_rows.argtypes = [vp, ctypes.POINTER(Rows), vp, ctypes.c_int64, vp]
    lib.ssb_restrict_slice.restype = ctypes.c_int
    lib.ssb_restrict_slice.argtypes = [vp, ctypes.POINTER(Rows), i32, i32, vp, ctypes.c_int64, vp]
    lib.ssb_shard_record_words.restype = ctypes.c_int64
    lib.ssb_shard_record_words.argtypes = [i32, i32]
    lib.ssb_shard_select.restype = ctypes.c_int
    lib.ssb_shard_select.argtypes = [vp, ctypes.POINTER(Rows), i32, i32, i32, vp, vp]
    lib.ssb_shard_merge.restype = ctypes.c_int
    lib.ssb_shard_merge.argtypes = [vp, ctypes.POINTER(Rows), i32, i32, i32, vp, vp]
    lib.ssb_lm_head_argmax.restype = ctypes.c_int
    lib.ssb_lm_head_argmax.argtypes = [vp, ctypes.POINTER(LmHead), vp]
    lib.ssb_sample_embed_rows.restype = ctypes.c_int
    lib.ssb_sample_embed_rows.argtypes = [vp, ctypes.POINTER(Rows), ctypes.POINTER(Embed), vp]
    lib.ssb_context_mask.restype = ctypes.c_int
    lib.ssb_context_mask.argtypes = [vp, vp, ctypes.c_int64, ctypes.POINTER(vp)]
    lib.ssb_dry_create.restype = ctypes.c_int
    lib.ssb_dry_create.argtypes = [vp, ctypes.POINTER(DryConfig), i32, vp, i32, ctypes.POINTER(vp)]
    lib.ssb_dry_destroy.restype = ctypes.c_int
    lib.ssb_dry_destroy.argtypes = [vp]
    lib.ssb_dry_update.restype = ctypes.c_int
    lib.ssb_dry_update.argtypes = [vp, vp, vp]
    lib.ssb_dry_penalties.restype = ctypes.c_int
    lib.ssb_dry_penalties.argtypes = [vp, i32, vp, vp, i32, ctypes.POINTER(i32), vp]
    lib.ssb_haru_shape_rows.restype = ctypes.c_int
    lib.ssb_haru_shape_rows.argtypes = [vp, ctypes.POINTER(HaruShape), vp, vp]
    _LIB = lib
    return lib


def _check(lib, status):
    if status != OK:
        raise SsbError(status, lib.ssb_last_error().decode())


def _dptr(t):
    """Device pointer of a torch tensor (or None)."""
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _hptr(a):
    return None if a is None else ctypes.c_void_p(a.ctypes.data)


class Sampler:
    """One engine context on one CUDA device."""

    def __init__(self, device: int = 0):
        self.lib = load_library()
        self.device = device
        ctx = ctypes.c_void_p()
        _check(self.lib, self.lib.ssb_context_create(device, ctypes.byref(ctx)))
        self.ctx = ctx

    def close(self):
        if self.ctx:
            self.lib.ssb_context_destroy(self.ctx)
            self.ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def reserve(self, max_rows: int, max_vocab: int):
        _check(self.lib, self.lib.ssb_context_reserve(self.ctx, max_rows, max_vocab))

    @staticmethod
    def _rows_struct(logits, p, history, history_len, mask, mask_kind, u, ids, status, row_params=None,
                     max_top_k=0, host=False):
        import torch  # noqa: F401  (only for dtype checks of device tensors)
        r = Rows()
        if host:
            x = logits
            r.dtype = BF16 if x.dtype == np.uint16 else F32
            r.rows, r.vocab = x.shape
            r.ld = x.strides[0] // x.itemsize
            r.logits = x.ctypes.data
            ptr = _hptr
        else:
            x = logits
            r.dtype = BF16 if str(x.dtype) == "torch.bfloat16" else F32
            if r.dtype == F32 and str(x.dtype) != "torch.float32":
                raise TypeError("logits must be float32 or bfloat16")
            r.rows, r.vocab = x.shape
            r.ld = x.stride(0)
            if x.stride(1) != 1:
                raise ValueError("logits rows must be contiguous")
            r.logits = x.data_ptr()
            ptr = _dptr
        r.max_top_k = max_top_k
        r.params = p if p is not None else params()
        r.row_params = ptr(row_params)
        if history is not None:
            r.history = ptr(history)
            r.history_ld = history.shape[1]
            r.history_len = ptr(history_len)
        if mask is not None and mask_kind != MASK_NONE:
            r.mask = ptr(mask)
            r.mask_ld = 0 if mask.ndim == 1 else mask.shape[1]
            r.mask_kind = mask_kind
        r.u = ptr(u)
        r.ids = ptr(ids)
        r.status = ptr(status)
        return r

    def sample(self, logits, p: Params | None = None, history=None, history_len=None, mask=None,
               mask_kind=MASK_NONE, u=None, row_params=None, max_top_k=0, ids=None, status=None, stream=None):
        """Device tensors in, device tensors out (asynchronous on `stream`, a torch.cuda.Stream or None)."""
        import torch
        b = logits.shape[0]
        if ids is None:
            ids = torch.empty(b, dtype=torch.int32, device=logits.device)
        if status is None:
            status = torch.empty(b, dtype=torch.int32, device=logits.device)
        r = self._rows_struct(logits, p, history, history_len, mask, mask_kind, u, ids, status, row_params, max_top_k)
        s = None if stream is None else ctypes.c_void_p(stream.cuda_stream)
        _check(self.lib, self.lib.ssb_sample_rows(self.ctx, ctypes.byref(r), s))
        return ids, status

    def sample_embed(self, logits, p: Params | None, table, out, u=None, history=None, history_len=None, mask=None,
                     mask_kind=MASK_NONE, ids=None, status=None, stream=None):
        """sample(), then out[r] = table[ids[r]] on the device (zeros for a refused row)."""
        import torch
        b = logits.shape[0]
        if ids is None:
            ids = torch.empty(b, dtype=torch.int32, device=logits.device)
        if status is None:
            status = torch.empty(b, dtype=torch.int32, device=logits.device)
        r = self._rows_struct(logits, p, history, history_len, mask, mask_kind, u, ids, status)
        e = Embed()
        e.table = table.data_ptr()
        e.table_rows, e.dim = table.shape
        e.ld = table.stride(0)
        e.dtype = BF16 if table.dtype == torch.bfloat16 else F32
        if out.dtype != table.dtype or out.shape[1] < e.dim:
            raise ValueError("out must have the table's dtype and at least its width")
        e.out = out.data_ptr()
        e.out_ld = out.stride(0)
        s = None if stream is None else ctypes.c_void_p(stream.cuda_stream)
        _check(self.lib, self.lib.ssb_sample_embed_rows(self.ctx, ctypes.byref(r), ctypes.byref(e), s))
        return ids, status

    def shard_select(self, logits_slice, p, col_offset: int, vocab_total: int, k_cap: int, records, history=None,
                     history_len=None, mask=None, mask_kind=MASK_NONE, row_params=None, stream=None):
        """Step 1 of the vocabulary-sharded draw on this slice (history: the rows' global ids; mask: the
        whole rows' words); records: uint64 device tensor of ssb_shard_record_words(rows, k_cap) words."""
        r = self._rows_struct(logits_slice, p, history, history_len, mask, mask_kind, None, None, None, row_params)
        s = None if stream is None else ctypes.c_void_p(stream.cuda_stream)
        _check(self.lib, self.lib.ssb_shard_select(self.ctx, ctypes.byref(r), col_offset, vocab_total, k_cap,
                                                  _dptr(records), s))

    def restrict_slice(self, logits_slice, p, col_offset: int, vocab_total: int, out, history=None, mask=None,
                       mask_kind=MASK_NONE, row_params=None, stream=None):
        """ssb_restrict_slice: the restricted logits of this slice into `out` (f32 [rows, >= width]); history
        holds the rows' global ids, mask the whole rows' words."""
        r = self._rows_struct(logits_slice, p, history, None, mask, mask_kind, None, None, None, row_params)
        s = None if stream is None else ctypes.c_void_p(stream.cuda_stream)
        _check(self.lib, self.lib.ssb_restrict_slice(self.ctx, ctypes.byref(r), col_offset, vocab_total, _dptr(out),
                                                    out.stride(0), s))
        return out

    def shard_merge(self, rows: int, p, vocab_total: int, world: int, k_cap: int, records, u=None, row_params=None,
                    ids=None, status=None, stream=None):
        """Step 2: ids and statuses of `rows` rows from the world ranks' records ([world][rows][k_cap + 1])."""
        import torch
        dev = records.device
        ids = torch.empty(rows, dtype=torch.int32, device=dev) if ids is None else ids
        status = torch.empty(rows, dtype=torch.int32, device=dev) if status is None else status
        r = Rows()
        r.rows, r.vocab, r.ld, r.dtype = rows, vocab_total, vocab_total, F32
        r.params = p if p is not None else params()
        r.row_params = _dptr(row_params)
        r.u, r.ids, r.status = _dptr(u), _dptr(ids), _dptr(status)
        s = None if stream is None else ctypes.c_void_p(stream.cuda_stream)
        _check(self.lib, self.lib.ssb_shard_merge(self.ctx, ctypes.byref(r), vocab_total, world, k_cap,
                                                 _dptr(records), s))
        return ids, status

    def lm_head_argmax(self, hidden, weight, ids=None, max_logit=None, status=None, stream=None):
        """ids[r] = first argmax over tokens of hidden[r] . weight[v] (bf16 in, fp32 accumulation), fused."""
        import torch
        rows, dim = hidden.shape
        if ids is None:
            ids = torch.empty(rows, dtype=torch.int32, device=hidden.device)
        h = LmHead()
        h.hidden, h.hidden_ld, h.rows, h.dim = hidden.data_ptr(), hidden.stride(0), rows, dim
        h.weight, h.weight_ld, h.vocab = weight.data_ptr(), weight.stride(0), weight.shape[0]
        h.dtype = BF16 if hidden.dtype == torch.bfloat16 and weight.dtype == torch.bfloat16 else F32
        h.ids, h.max_logit, h.status = ids.data_ptr(), _dptr(max_logit), _dptr(status)
        s = None if stream is None else ctypes.c_void_p(stream.cuda_stream)
        _check(self.lib, self.lib.ssb_lm_head_argmax(self.ctx, ctypes.byref(h), s))
        return ids

    def candidates(self, logits, p: Params | None = None, history=None, history_len=None, mask=None,
                   mask_kind=MASK_NONE, u=None, row_params=None, max_top_k=0, cap=64, processed=True, stream=None):
        """The parity export: ids, status, tokens [B,cap], weights [B,cap], count [B], processed [B,V]."""
        import torch
        b, v = logits.shape
        dev = logits.device
        ids = torch.empty(b, dtype=torch.int32, device=dev)
        status = torch.empty(b, dtype=torch.int32, device=dev)
        tokens = torch.full((b, max(cap, 1)), -1, dtype=torch.int32, device=dev)
        weights = torch.zeros((b, max(cap, 1)), dtype=torch.float64, device=dev)
        count = torch.zeros(b, dtype=torch.int32, device=dev)
        proc = torch.empty((b, v), dtype=torch.float32, device=dev) if processed else None
        r = self._rows_struct(logits, p, history, history_len, mask, mask_kind, u, ids, status, row_params, max_top_k)
        s = None if stream is None else ctypes.c_void_p(stream.cuda_stream)
        _check(self.lib, self.lib.ssb_candidates_rows(self.ctx, ctypes.byref(r), cap, _dptr(tokens), _dptr(weights),
                                                     _dptr(count), _dptr(proc), s))
        return ids, status, tokens, weights, count, proc

    def restrict(self, logits, p: Params | None = None, history=None, history_len=None, mask=None,
                 mask_kind=MASK_NONE, row_params=None, out=None, stream=None):
        """The restricted logits (penalties and mask, before the temperature) as f32 [B, V] on the
        device: the reference's restricted() for a batch (ssb_restrict_rows)."""
        import torch
        b, v = logits.shape
        if out is None:
            out = torch.empty((b, v), dtype=torch.float32, device=logits.device)
        elif out.dtype != torch.float32 or out.shape[0] != b or out.shape[1] < v or out.stride(1) != 1:
            raise ValueError("out must be float32 [B, >= V] with contiguous rows")
        r = self._rows_struct(logits, p, history, history_len, mask, mask_kind, None, None, None, row_params)
        s = None if stream is None else ctypes.c_void_p(stream.cuda_stream)
        _check(self.lib, self.lib.ssb_restrict_rows(self.ctx, ctypes.byref(r), _dptr(out), out.stride(0), s))
        return out

    def sample_host(self, logits, p: Params | None = None, history=None, history_len=None, mask=None,
                    mask_kind=MASK_NONE, u=None, row_params=None, max_top_k=0, ids=None, status=None, stream=None):
        """Host (numpy) buffers in and out; copies happen inside the call, which waits for the result."""
        b = logits.shape[0]
        ids = np.empty(b, np.int32) if ids is None else ids
        status = np.empty(b, np.int32) if status is None else status
        r = self._rows_struct(logits, p, history, history_len, mask, mask_kind, u, ids, status, row_params,
                              max_top_k, host=True)
        s = None if stream is None else ctypes.c_void_p(stream.cuda_stream)
        _check(self.lib, self.lib.ssb_sample_host(self.ctx, ctypes.byref(r), s))
        return ids, status


class Dry:
    """The DRY state of `streams` Haru text streams on the device (haru::Dry, haru/sampler.h:49-69)."""

    def __init__(self, sampler: "Sampler", config: DryConfig, streams: int, exempt=()):
        self.lib = sampler.lib
        self.streams = streams
        ex = np.ascontiguousarray(np.asarray(exempt, np.int32))
        h = ctypes.c_void_p()
        _check(self.lib, self.lib.ssb_dry_create(sampler.ctx, ctypes.byref(config), streams,
                                                 _hptr(ex) if len(ex) else None, len(ex), ctypes.byref(h)))
        self.h = h

    def update(self, tokens, stream=None):
        """Dry::update(tokens[s]) for every stream s; tokens: int32 device tensor [streams] (< 0: skip)."""
        s = None if stream is None else ctypes.c_void_p(stream.cuda_stream)
        _check(self.lib, self.lib.ssb_dry_update(self.h, _dptr(tokens), s))

    def penalties(self, s: int, cap: int = 1024, stream=None):
        """Dry::penalties() of stream s: (tokens int32, penalties float64) by rising token."""
        t = np.empty(cap, np.int32)
        v = np.empty(cap, np.float64)
        n = ctypes.c_int32(0)
        st = None if stream is None else ctypes.c_void_p(stream.cuda_stream)
        _check(self.lib, self.lib.ssb_dry_penalties(self.h, s, _hptr(t), _hptr(v), cap, ctypes.byref(n), st))
        k = min(n.value, cap)
        return t[:k].copy(), v[:k].copy()

    def close(self):
        if self.h:
            self.lib.ssb_dry_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def haru_shape(sampler: "Sampler", logits, silent, pad: int, eop: int, eos: int, eop_bias: float = 0.0,
               must_speak=None, dry: Dry | None = None, stream=None):
    """shape_logits() (haru/sampler.cpp:116-124) on f32 device rows [rows, V], in place."""
    h = HaruShape()
    h.logits = logits.data_ptr()
    h.rows, h.vocab = logits.shape
    h.ld = logits.stride(0)
    h.silent = silent.data_ptr()
    h.silent_ld = silent.stride(0)
    h.pad, h.eop, h.eos = pad, eop, eos
    h.eop_bias = eop_bias
    h.must_speak = _dptr(must_speak)
    s = None if stream is None else ctypes.c_void_p(stream.cuda_stream)
    _check(sampler.lib, sampler.lib.ssb_haru_shape_rows(sampler.ctx, ctypes.byref(h), dry.h if dry else None, s))
