"""Failure detection without a GPU fault: the top-k kernel's bounded waits.

The wait-limit test library (libspeech_sampler_b200_waittest.so, the engine's sources built with
SSB_WAIT_TEST: waits give up after about 2 ms, and row 0's first refill of the shared-memory ring is
never issued) runs a config-4 batch whose row 0 streams through one CTA. Row 0's consumers wait for a
stage that nothing fills; the wait runs out, the row must come back as SSB_ROW_DEVICE_TIMEOUT, every
other row must still equal the oracle, the kernel must neither fault nor hang, and afterwards both the
same library (on rows its planted gap does not reach) and the product library must serve normal calls
on the same device."""
import ctypes
import os

import numpy as np
import pytest

import speech_sampler as ss
import speech_workloads as wl
from oracle import params

pytestmark = pytest.mark.gpu
WAITTEST = os.path.join(os.path.dirname(ss.LIB_PATH), "libspeech_sampler_b200_waittest.so")


def _lib(path):
    lib = ctypes.CDLL(path)
    vp = ctypes.c_void_p
    lib.ssb_context_create.restype = ctypes.c_int
    lib.ssb_context_create.argtypes = [ctypes.c_int32, ctypes.POINTER(vp)]
    lib.ssb_context_destroy.argtypes = [vp]
    lib.ssb_sample_rows.restype = ctypes.c_int
    lib.ssb_sample_rows.argtypes = [vp, ctypes.POINTER(ss.Rows), vp]
    lib.ssb_last_error.restype = ctypes.c_char_p
    return lib


def test_wait_that_runs_out_reports_device_timeout(oracle):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    assert os.path.exists(WAITTEST), "the wait-limit test library is not built (speech_build.py builds it)"
    torch.cuda.set_device(0)
    lib = _lib(WAITTEST)
    ctx = ctypes.c_void_p()
    assert lib.ssb_context_create(0, ctypes.byref(ctx)) == ss.OK
    try:
        c = wl.config4(rows=256)  # one CTA per row: row 0 streams all 19 stages through the ring
        x = torch.from_numpy(c["logits_bf16"]).view(torch.bfloat16).cuda()
        h = torch.from_numpy(c["history"]).cuda()
        u = torch.from_numpy(c["u"]).cuda()
        p = ss.params(**c["params"])
        want, wst, _ = oracle.sample_rows(c["logits_bf16"], params(**c["params"]), history=c["history"], u=c["u"])
        for call in range(2):
            ids = torch.full((256,), -7, dtype=torch.int32, device="cuda")
            st = torch.full((256,), -7, dtype=torch.int32, device="cuda")
            r = ss.Sampler._rows_struct(x, p, h, None, None, ss.MASK_NONE, u, ids, st)
            assert lib.ssb_sample_rows(ctx, ctypes.byref(r), None) == ss.OK, lib.ssb_last_error()
            torch.cuda.synchronize()  # raises if the kernel faulted
            got_ids, got_st = ids.cpu().numpy(), st.cpu().numpy()
            assert got_st[0] == ss.ROW_DEVICE_TIMEOUT and got_ids[0] == -1, (call, got_st[0], got_ids[0])
            assert np.array_equal(got_st[1:], wst[1:]) and np.array_equal(got_ids[1:], want[1:]), call
        # the same library on short rows (no refill is skipped) answers normally
        c2 = wl.config2(steps=4)
        x2 = torch.from_numpy(c2["logits"]).cuda()
        ids = torch.empty(4, dtype=torch.int32, device="cuda")
        st = torch.empty(4, dtype=torch.int32, device="cuda")
        r = ss.Sampler._rows_struct(x2, ss.params(**c2["params"]), torch.from_numpy(c2["history"]).cuda(), None, None,
                                    ss.MASK_NONE, torch.from_numpy(c2["u"]).cuda(), ids, st)
        assert lib.ssb_sample_rows(ctx, ctypes.byref(r), None) == ss.OK
        torch.cuda.synchronize()
        want2, _, _ = oracle.sample_rows(c2["logits"], params(**c2["params"]), history=c2["history"], u=c2["u"])
        assert np.array_equal(ids.cpu().numpy(), want2) and np.all(st.cpu().numpy() == 0)
    finally:
        lib.ssb_context_destroy(ctx)
    # the product library on the same device, after the timed-out launch
    s = ss.Sampler(0)
    try:
        c = wl.config4(rows=8)
        x = torch.from_numpy(c["logits_bf16"]).view(torch.bfloat16).cuda()
        ids, st = s.sample(x, ss.params(**c["params"]), torch.from_numpy(c["history"]).cuda(),
                           u=torch.from_numpy(c["u"]).cuda())
        torch.cuda.synchronize()
        want, wst, _ = oracle.sample_rows(c["logits_bf16"], params(**c["params"]), history=c["history"], u=c["u"])
        assert np.array_equal(ids.cpu().numpy(), want) and np.array_equal(st.cpu().numpy(), wst)
    finally:
        s.close()
