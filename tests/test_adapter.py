"""The C++ call-site wrapper (include/speech_sampler_b200.hpp) against the reference it replaces. The
check library (oracle/ref_shim/adapter_check.cpp, built into oracle/_ref/libadapter_check.so against the
reference's own headers and sampler sources) runs each call through the reference and through the
wrapper; these tests require identical outcomes: the same id (integers: zero tolerance), or the same
exception — type, Fault, input name and message — and, over a seeded talker loop, the same ids at every
frame and generators that end in the same state (the rng overload draws only where a row draws)."""
import ctypes
import os

import numpy as np
import pytest

import speech_sampler as ss
import speech_workloads as wl

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ADAPTER_SO = os.path.join(ROOT, "oracle", "_ref", "libadapter_check.so")
FAULT_OUT_OF_RANGE, FAULT_DEVICE = 1, 3  # Fault::OutOfRange, Fault::Device (src/common/error.h:8-21)


class Outcome(ctypes.Structure):
    _fields_ = [("id", ctypes.c_int32), ("kind", ctypes.c_int32), ("fault", ctypes.c_int32),
                ("input", ctypes.c_char * 64), ("message", ctypes.c_char * 448)]

    def key(self):
        return (self.id, self.kind, self.fault, self.input, self.message)


def _lib():
    if not os.path.exists(ADAPTER_SO):
        pytest.skip("oracle/_ref/libadapter_check.so is not built (oracle/Makefile adapter; needs the reference)")
    lib = ctypes.CDLL(ADAPTER_SO)
    f32p, i32p = ctypes.POINTER(ctypes.c_float), ctypes.POINTER(ctypes.c_int32)
    op = ctypes.POINTER(Outcome)
    lib.adapter_sample.restype = None
    lib.adapter_sample.argtypes = [f32p, ctypes.c_int32, ctypes.POINTER(ss.Params), i32p, ctypes.c_int32,
                                   ctypes.POINTER(ctypes.c_uint8), ctypes.c_int32, ctypes.c_double, op, op]
    for name in ("adapter_haru", "adapter_drama3"):
        f = getattr(lib, name)
        f.restype = None
        f.argtypes = [f32p, ctypes.c_int32, ctypes.c_float, ctypes.c_int32, ctypes.c_float, ctypes.c_double, op, op]
    lib.adapter_talker_loop.restype = ctypes.c_int64
    lib.adapter_talker_loop.argtypes = [f32p, ctypes.c_int64, ctypes.c_int32, ctypes.POINTER(ss.Params),
                                        ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                        ctypes.c_uint64, ctypes.c_int32, i32p, i32p, i32p]
    lib.adapter_last_message.restype = ctypes.c_char_p
    return lib


def _p(a, t):
    return None if a is None else a.ctypes.data_as(ctypes.POINTER(t))


def test_adapter_library_exports():
    """CPU: the check library loads (with the engine it links) and exports its entry points."""
    lib = _lib()
    for name in ("adapter_sample", "adapter_haru", "adapter_drama3", "adapter_talker_loop", "adapter_last_message"):
        assert hasattr(lib, name)


def test_wrapper_header_declares_reference_signatures():
    """CPU: the wrapper keeps the reference's call signatures (qwen3-tts/sampler.h:61-71)."""
    text = open(os.path.join(ROOT, "include", "speech_sampler_b200.hpp")).read()
    assert "const std::vector<bool> & banned, double u)" in text
    assert "const std::vector<bool> & banned, std::mt19937_64 & rng)" in text
    assert "p.greedy ? 0.0 : uniform(rng)" in text


def _sample(lib, x, p, history=None, banned=None, u=0.5):
    a, r = Outcome(), Outcome()
    x = np.ascontiguousarray(x, np.float32)
    h = None if history is None else np.ascontiguousarray(history, np.int32)
    b = None if banned is None else np.ascontiguousarray(banned, np.uint8)
    lib.adapter_sample(_p(x, ctypes.c_float), len(x), ctypes.byref(p), _p(h, ctypes.c_int32),
                       0 if h is None else len(h), _p(b, ctypes.c_uint8), 0 if b is None else len(b), float(u),
                       ctypes.byref(a), ctypes.byref(r))
    return a, r


@pytest.mark.gpu
def test_wrapper_rethrows_the_references_exceptions():
    lib = _lib()
    # checks/qwen3-tts/qwen3-tts-sampler-check.cpp:70-91: a penalty of 1e-40 on logits 1 and 2 in the history
    x = np.array([1.0, 2.0], np.float32)
    for greedy in (True, False):
        a, r = _sample(lib, x, ss.params(greedy=greedy, repetition_penalty=1e-40), history=[0, 1])
        assert r.kind == 1 and r.fault == FAULT_OUT_OF_RANGE and r.input == b"repetition_penalty"
        assert a.key() == r.key()
    # a temperature that pushes the largest logit beyond a float
    a, r = _sample(lib, np.array([1.0, 30.0, 2.0], np.float32), ss.params(temperature=1e-38, top_k=2))
    assert r.kind == 1 and r.input == b"temperature" and a.key() == r.key()
    # every token banned
    a, r = _sample(lib, np.zeros(8, np.float32), ss.params(top_k=3), banned=np.ones(8, np.uint8))
    assert r.kind == 2 and a.key() == r.key()
    assert b"finite" in r.message
    # Haru: NaN and +inf are the device's Error; an overflowing temperature; T <= 0 takes the first max
    for fam in (lib.adapter_haru, lib.adapter_drama3):
        y = np.linspace(-2, 2, 64).astype(np.float32)
        y[9] = np.nan
        a, r = Outcome(), Outcome()
        fam(_p(y, ctypes.c_float), len(y), 0.8, 10, 0.9, 0.3, ctypes.byref(a), ctypes.byref(r))
        assert r.kind == 1 and r.fault == FAULT_DEVICE and a.key() == r.key()
        big = (np.linspace(-2, 2, 64) * 1e37).astype(np.float32)
        fam(_p(big, ctypes.c_float), len(big), 1e-30, 10, 0.9, 0.3, ctypes.byref(a), ctypes.byref(r))
        assert r.kind == 1 and r.input == b"temperature" and a.key() == r.key()
    z = np.zeros(100, np.float32)
    z[[7, 70]] = 1.0
    a, r = Outcome(), Outcome()
    lib.adapter_haru(_p(z, ctypes.c_float), len(z), 0.0, 10, 0.9, 0.99, ctypes.byref(a), ctypes.byref(r))
    assert r.kind == 0 and r.id == 7 and a.key() == r.key()


@pytest.mark.gpu
def test_wrapper_ids_equal_the_references():
    lib = _lib()
    rng = np.random.default_rng(12)
    for trial in range(60):
        n = int(rng.choice([64, 2048, 3072, 151936]))
        x = (rng.standard_normal(n) * 2).astype(np.float32)
        p = ss.params(greedy=bool(rng.random() < 0.2), temperature=float(rng.choice([0.7, 0.9, 1.3])),
                      top_k=int(rng.choice([0, 1, 50, 200])), top_p=float(rng.choice([1.0, 0.9, 0.5])),
                      repetition_penalty=float(rng.choice([1.0, 1.05, 1.3])))
        if n > 8192 and p.top_k == 0:
            p.top_k = 50
        h = rng.integers(0, n, size=int(rng.integers(0, 512))).astype(np.int32)
        banned = (rng.random(n) < 0.05).astype(np.uint8)
        a, r = _sample(lib, x, p, h, banned, float(rng.random()))
        assert r.kind == 0 and a.key() == r.key(), (trial, a.id, r.id)
        t, k, tp = float(rng.choice([0.0, 0.7, 1.5])), int(rng.choice([0, 25, 500])), float(rng.choice([1.0, 0.9]))
        if n > 8192:
            k = 25
        u = float(rng.random())
        for fam in (lib.adapter_haru, lib.adapter_drama3):
            fam(_p(x, ctypes.c_float), n, t, k, tp, u, ctypes.byref(a), ctypes.byref(r))
            assert r.kind == 0 and a.key() == r.key(), (trial, fam, a.id, r.id)


@pytest.mark.gpu
@pytest.mark.parametrize("mode", [0, 1])
@pytest.mark.parametrize("greedy", [False, True])
def test_talker_loop_with_rng(mode, greedy):
    """2048 frames of config 2's talker (3072 codes, T 0.9, k 50, p 1, penalty 1.05) with the
    suppress mask of Generation::banned (the last 1024 ids but the end of speech 2150, the end of speech
    before frame 2) and the code predictor's 15 draws per frame between the talker's: the wrapper's
    ids equal the reference's at every frame and both generators end in the same state."""
    lib = _lib()
    steps, vocab = 2048, wl.TALKER_VOCAB
    x = (np.random.default_rng(3).standard_normal((steps, vocab)) * 2).astype(np.float32)
    x[:, 2150] += 3.0  # the end of speech is likely once allowed
    p = ss.params(greedy=greedy, temperature=0.9, top_k=50, top_p=1.0, repetition_penalty=1.05)
    ids_a = np.full(steps, -7, np.int32)
    ids_r = np.full(steps, -8, np.int32)
    eq = ctypes.c_int32(0)
    rc = lib.adapter_talker_loop(_p(x, ctypes.c_float), steps, vocab, ctypes.byref(p), 2150, 1024, 2, 15,
                                 20250101, mode, _p(ids_a, ctypes.c_int32), _p(ids_r, ctypes.c_int32),
                                 ctypes.byref(eq))
    assert rc == 0, lib.adapter_last_message()
    assert np.array_equal(ids_a, ids_r)
    assert eq.value == 1
    assert np.all(ids_r[:2] != 2150) and np.all(ids_r[ids_r != 2150] < vocab - 1024)
