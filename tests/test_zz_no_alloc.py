"""ssb_sample_rows_noalloc — sampling for callers that cannot allocate device memory (a runtime that
owns every device buffer through its own pool, or a decode loop that must not call cudaMalloc). It
uses a fixed scratch array inside the library instead of a context's allocations, so its answers must
be exactly those of ssb_sample_rows, and those of the oracle restatement (token ids and statuses are
integers: the tolerance is zero), on two calls in a row (the shared array keeps the previous call's
contents). This file is collected last so that a run stopping at the first failure has run every
other test; it also passes alone in a fresh process, where its first call performs the per-device
set-up."""
import ctypes

import numpy as np
import pytest

import speech_sampler as ss
import speech_workloads as wl
from oracle import Oracle, params as oparams

pytestmark = pytest.mark.gpu


def _noalloc(lib):
    f = lib.ssb_sample_rows_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.POINTER(ss.Rows), ctypes.c_void_p]
    return f


def _cases():
    """(name, logits host array, params, history, mask, mask kind, u): batches that make the kernel
    split rows over several CTAs (the scratch's users) and one that does not."""
    c4 = wl.config4(rows=8)
    c1 = wl.config1(rows=3)
    big = wl.config4(rows=256)
    return [
        ("config4 8 rows (split rows, bf16, penalties)", c4["logits_bf16"], ss.params(**c4["params"]), c4["history"],
         None, ss.MASK_NONE, c4["u"]),
        ("config1 3 rows (greedy, ban mask, fp32)", c1["logits"], ss.params(greedy=True), None, c1["mask"],
         ss.MASK_BAN, None),
        ("config4 256 rows (one CTA per row)", big["logits_bf16"], ss.params(**big["params"]), big["history"], None,
         ss.MASK_NONE, big["u"]),
    ]


def test_noalloc_matches_sample_rows_twice():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.set_device(0)
    lib = ss.load_library()
    noalloc = _noalloc(lib)
    sampler = ss.Sampler(0)
    oracle = Oracle()
    try:
        for name, x, p, hist, mask, kind, u in _cases():
            xt = torch.from_numpy(x)
            xt = (xt.view(torch.bfloat16) if x.dtype == np.uint16 else xt).cuda()
            h = None if hist is None else torch.from_numpy(hist).cuda()
            m = None if mask is None else torch.from_numpy(mask.view(np.int32)).cuda()
            uu = None if u is None else torch.from_numpy(u).cuda()
            want_ids, want_st = sampler.sample(xt, p, h, None, m, kind, uu)
            torch.cuda.synchronize()
            op = oparams(greedy=bool(p.greedy), temperature=p.temperature, top_k=p.top_k, top_p=p.top_p,
                         repetition_penalty=p.repetition_penalty, presence_penalty=p.presence_penalty,
                         frequency_penalty=p.frequency_penalty)
            o_ids, o_st, _ = oracle.sample_rows(x, op, history=hist, mask=mask, mask_kind=kind, u=u)
            for call in range(2):
                ids = torch.full((x.shape[0],), -7, dtype=torch.int32, device="cuda")
                st = torch.full((x.shape[0],), -7, dtype=torch.int32, device="cuda")
                r = ss.Sampler._rows_struct(xt, p, h, None, m, kind, uu, ids, st)
                got = noalloc(ctypes.byref(r), None)
                assert got == ss.OK, (name, call, lib.ssb_last_error().decode())
                torch.cuda.synchronize()
                assert torch.equal(ids, want_ids), (name, call)
                assert torch.equal(st, want_st), (name, call)
                assert np.array_equal(ids.cpu().numpy(), o_ids) and np.array_equal(st.cpu().numpy(), o_st), (name, call)
    finally:
        sampler.close()


def test_noalloc_refuses_beyond_its_limits():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    lib = ss.load_library()
    noalloc = _noalloc(lib)
    x = torch.zeros((2, 151936), dtype=torch.float32, device="cuda")
    ids = torch.empty(2, dtype=torch.int32, device="cuda")
    st = torch.empty(2, dtype=torch.int32, device="cuda")
    u = torch.zeros(2, dtype=torch.float64, device="cuda")
    r = ss.Sampler._rows_struct(x, ss.params(top_k=500), None, None, None, ss.MASK_NONE, u, ids, st)
    assert noalloc(ctypes.byref(r), None) == ss.OUT_OF_RANGE
    assert "top-k of at most 128" in lib.ssb_last_error().decode()
    small = torch.zeros((2, 3072), dtype=torch.float32, device="cuda")
    r = ss.Sampler._rows_struct(small, ss.params(top_k=50), None, None, None, ss.MASK_NONE, u, ids, st)
    assert noalloc(ctypes.byref(r), None) == ss.OUT_OF_RANGE
    assert "more than 8192 tokens" in lib.ssb_last_error().decode()
