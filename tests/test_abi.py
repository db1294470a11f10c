"""The C-ABI library: it is built, loads, exports every function include/speech_sampler_b200.h
declares, and refuses bad arguments on the host before touching a device. CPU only (no kernel runs)."""
import ctypes
import os

import numpy as np
import pytest

import speech_sampler as ss


@pytest.fixture(scope="module")
def lib():
    import speech_build
    speech_build.build()
    return ss.load_library()


def test_exports_every_declared_symbol(lib):
    declared = ss.header_symbols()
    assert len(declared) >= 8
    import subprocess
    out = subprocess.run(["nm", "-D", "--defined-only", ss.LIB_PATH], capture_output=True, text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = [s for s in declared if s not in exported]
    assert not missing, missing
    extra = sorted(s for s in exported if s.startswith("ssb_") and s not in declared)
    assert not extra, f"exported but undeclared: {extra}"
    for s in declared:
        getattr(lib, s)  # resolvable through ctypes too


def test_version_and_struct_layout(lib):
    assert lib.ssb_version().decode().count(".") == 2
    assert ctypes.sizeof(ss.Params) == 32
    assert ctypes.sizeof(ss.Rows) == 144
    assert ss.Rows.params.offset == 32 and ss.Rows.status.offset == 136


def _rows(**kw):
    r = ss.Rows()
    r.logits = 0x1000
    r.ld = 8
    r.dtype = ss.F32
    r.rows = 2
    r.vocab = 8
    r.params = ss.params(greedy=True)
    r.ids = 0x2000
    r.status = 0x3000
    for k, v in kw.items():
        setattr(r, k, v)
    return r


@pytest.mark.parametrize("field,value,status,needle", [
    ("rows", -1, ss.INVALID_ARGUMENT, "negative"),
    ("vocab", 0, ss.INVALID_ARGUMENT, "vocab"),
    ("vocab", (1 << 24) + 1, ss.OUT_OF_RANGE, "SSB_MAX_VOCAB"),
    ("ld", 4, ss.INVALID_ARGUMENT, "ld"),
    ("dtype", 7, ss.INVALID_ARGUMENT, "dtype"),
    ("mask_kind", 3, ss.INVALID_ARGUMENT, "mask_kind"),
    ("reserved", 1, ss.INVALID_ARGUMENT, "reserved"),
    ("params", ss.params(flavor=3), ss.INVALID_ARGUMENT, "flavor"),
    ("logits", None, ss.INVALID_ARGUMENT, "logits"),
    ("ids", None, ss.INVALID_ARGUMENT, "ids"),
])
def test_bad_arguments_refused_on_host(lib, field, value, status, needle):
    r = _rows(**{field: value})
    got = lib.ssb_sample_rows(None, ctypes.byref(r), None)
    assert got == status
    assert needle in lib.ssb_last_error().decode()


def test_semantic_refusals(lib):
    r = _rows(params=ss.params(temperature=0.9, top_k=50))  # a draw without u
    assert lib.ssb_sample_rows(None, ctypes.byref(r), None) == ss.INVALID_ARGUMENT
    assert "u is required" in lib.ssb_last_error().decode()
    r = _rows(mask_kind=ss.MASK_BAN)  # a mask kind without a mask
    assert lib.ssb_sample_rows(None, ctypes.byref(r), None) == ss.INVALID_ARGUMENT
    r = _rows(vocab=151936, ld=151936, params=ss.params(top_k=0), u=0x4000)  # every token kept: valid, no ctx
    assert lib.ssb_sample_rows(None, ctypes.byref(r), None) == ss.INVALID_ARGUMENT
    assert "ctx" in lib.ssb_last_error().decode()
    r = _rows(vocab=151936, ld=151936, history=0x5000, history_ld=9000)
    assert lib.ssb_sample_rows(None, ctypes.byref(r), None) == ss.OUT_OF_RANGE
    assert "SSB_MAX_STREAM_HISTORY" in lib.ssb_last_error().decode()
    r = _rows()  # a valid batch with no context
    assert lib.ssb_sample_rows(None, ctypes.byref(r), None) == ss.INVALID_ARGUMENT
    assert "ctx" in lib.ssb_last_error().decode()
    assert lib.ssb_candidates_rows(None, ctypes.byref(r), -1, None, None, None, None, None) == ss.INVALID_ARGUMENT


def test_no_device_fails_loudly(lib):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    ctx = ctypes.c_void_p()
    st = lib.ssb_context_create(0, ctypes.byref(ctx))
    assert st in (ss.DEVICE, ss.INVALID_ARGUMENT) and not ctx.value
    with pytest.raises(ss.SsbError):
        ss.Sampler(0)


def test_nccl_library_exports():
    """The NCCL host library of the vocabulary-sharded draw loads (with the engine and libnccl) and exports
    every function its header declares."""
    import os
    import re
    import speech_vocab_shard as vs
    lib = vs.load_nccl_library()
    header = os.path.join(os.path.dirname(ss.HEADER), "speech_sampler_b200_nccl.h")
    names = re.findall(r"SSB_API\s+[^;(]*?\b(ssb_\w+)\s*\(", open(header).read())
    assert len(names) == 6
    for n in names:
        assert hasattr(lib, n), n
