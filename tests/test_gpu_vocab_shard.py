"""Vocabulary-sharded sampling (speech_vocab_shard): a row's columns split into slices, each restricted on
its own through the C ABI, laid side by side and drawn from. The ids and statuses must equal the whole-row
engine's exactly (the same engine, the same restricted logits, the same u). The slices run one after
another on one GPU here; the NCCL exchange itself is checked on CPU ranks (test_multirank.py)."""
import numpy as np
import pytest

import speech_sampler as ss
import speech_vocab_shard as vs
import speech_workloads as wl

from test_gpu_parity import dev

pytestmark = pytest.mark.gpu


def whole_and_sliced(engine, x, world, p, history=None, mask=None, mask_kind=ss.MASK_NONE, u=None):
    import torch
    ids_w, st_w = engine.sample(x, p, history, None, mask, mask_kind, u)
    ids_s, st_s = vs.sample_slices_on_one_device(engine, x, world, p, history, mask, mask_kind, u)
    torch.cuda.synchronize()
    return (int(ids_w.item()), int(st_w.item())), (int(ids_s.item()), int(st_s.item()))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_config5_rows(engine, world):
    import torch
    c = wl.config5(rows=3, density=0.01)
    p = ss.params(**c["params"])
    for r in range(3):
        x = dev(c["logits"][r:r + 1])
        m = dev(c["mask"][r:r + 1].view(np.int32))
        u = dev(c["u"][r:r + 1])
        whole, sliced = whole_and_sliced(engine, x, world, p, mask=m, mask_kind=ss.MASK_ALLOW, u=u)
        assert whole == sliced and whole[1] == ss.ROW_OK


@pytest.mark.parametrize("world", [2, 8])
def test_config4_rows_with_history(engine, world):
    import torch
    c = wl.config4(rows=3)
    p = ss.params(**c["params"])
    for r in range(3):
        x = dev(c["logits_bf16"][r:r + 1], torch.bfloat16)
        h = dev(c["history"][r:r + 1])
        u = dev(c["u"][r:r + 1])
        whole, sliced = whole_and_sliced(engine, x, world, p, history=h, u=u)
        assert whole == sliced and whole[1] == ss.ROW_OK
        # greedy and a repetition penalty, same row
        pg = ss.params(greedy=True, repetition_penalty=1.3)
        whole, sliced = whole_and_sliced(engine, x, world, pg, history=h, u=u)
        assert whole == sliced and whole[1] == ss.ROW_OK


def test_statuses_decided_on_the_whole_row(engine):
    """NaN in one slice, every column banned, +inf with a repetition penalty: the whole row's status."""
    rng = np.random.default_rng(61)
    v = 151936
    u = dev(np.array([0.4]))
    p = ss.params(temperature=1.0, top_k=20, top_p=0.9, repetition_penalty=1.1)
    x = rng.standard_normal((1, v), dtype=np.float32)
    nan_row = x.copy()
    nan_row[0, 100000] = np.nan
    inf_row = x.copy()
    inf_row[0, 5] = np.inf
    ban_all = wl.pack_mask(np.ones((1, v), bool))
    cases = [(nan_row, None, ss.ROW_NON_FINITE_INPUT), (inf_row, None, ss.ROW_PENALTY_OVERFLOW),
             (x, ban_all, ss.ROW_NO_FINITE_LOGIT)]
    for row, mask, want in cases:
        m = None if mask is None else dev(mask.view(np.int32))
        whole, sliced = whole_and_sliced(engine, dev(row), 4, p, mask=m,
                                         mask_kind=ss.MASK_BAN if mask is not None else ss.MASK_NONE, u=u)
        assert whole == sliced and whole[1] == want


# ---------------------------------------------------------------- the candidate exchange (top-k rows)
def _exchange_vs_whole(engine, x, world, p, k_cap, history=None, mask=None, mask_kind=ss.MASK_NONE, u=None,
                       row_params=None, max_top_k=0):
    import torch
    ids_w, st_w = engine.sample(x, p, history, None, mask, mask_kind, u, row_params, max_top_k)
    ids_s, st_s = vs.sample_topk_on_one_device(engine, x, world, p, history, mask, mask_kind, u, k_cap, row_params)
    torch.cuda.synchronize()
    return ids_w.cpu().numpy(), st_w.cpu().numpy(), ids_s.cpu().numpy(), st_s.cpu().numpy()


@pytest.mark.parametrize("world", [2, 3, 8])
def test_exchange_config4_batch(engine, world):
    """Config 4's rows (bf16, 1024 history ids, repetition/presence/frequency penalties, top-k 40, top-p
    0.95) as `world` slices: each slice's 64 best composites, merged: ids and statuses equal the
    whole-row engine's on all 64 rows."""
    c = wl.config4(rows=64)
    import torch
    x = dev(c["logits_bf16"], torch.bfloat16)
    p = ss.params(**c["params"])
    iw, sw, i_s, s_s = _exchange_vs_whole(engine, x, world, p, 64, dev(c["history"]), u=dev(c["u"]))
    assert np.array_equal(sw, s_s) and np.all(sw == ss.ROW_OK)
    assert np.array_equal(iw, i_s)


@pytest.mark.parametrize("world", [2, 4])
def test_exchange_talker_and_greedy_masked(engine, world):
    """Talker rows (3072 codes, k 50, penalty 1.05 over 512 ids) and greedy rows with a ban mask (the ASR
    suppress mask at 151936 tokens), k_cap 64 and 1."""
    import torch
    t = wl.config2(steps=16)
    p2 = ss.params(**t["params"])
    iw, sw, i_s, s_s = _exchange_vs_whole(engine, dev(t["logits"]), world, p2, 64, dev(t["history"]), u=dev(t["u"]))
    assert np.array_equal(sw, s_s) and np.array_equal(iw, i_s)
    c1 = wl.config1(rows=8)
    m = dev(c1["mask"].view(np.int32))
    iw, sw, i_s, s_s = _exchange_vs_whole(engine, dev(c1["logits"]), world, ss.params(greedy=True), 1, mask=m,
                                          mask_kind=ss.MASK_BAN)
    assert np.array_equal(sw, s_s) and np.array_equal(iw, i_s)


def test_exchange_statuses_and_row_params(engine):
    """NaN, +inf with a penalty, every token banned, an overflowing temperature, a greedy row and a row
    keeping more than k_cap (top-k 0: INVALID_ROW) among per-row settings."""
    import torch
    rng = np.random.default_rng(17)
    V = 20000
    x = (rng.standard_normal((6, V)) * 2).astype(np.float32)
    x[0, 1234] = np.nan
    x[1, 50] = np.inf
    x[3, :] *= np.float32(1e30)
    hist = np.full((6, 4), -1, np.int32)
    hist[1, 0] = 50
    ban = np.zeros((6, V), bool)
    ban[2, :] = True
    mask = wl.pack_mask(ban)
    plist = [ss.params(temperature=0.9, top_k=40), ss.params(temperature=0.9, top_k=40, repetition_penalty=1.3),
             ss.params(temperature=0.9, top_k=40), ss.params(temperature=1e-30, top_k=40),
             ss.params(greedy=True, repetition_penalty=1.3), ss.params(temperature=0.9, top_k=0)]
    u = rng.random(6)
    rp = dev(ss.params_array(plist).view(np.uint8)).view(torch.int32)
    iw, sw, i_s, s_s = _exchange_vs_whole(engine, dev(x), 4, plist[0], 64, dev(hist), dev(mask.view(np.int32)),
                                          ss.MASK_BAN, dev(u), rp, max_top_k=0)
    assert list(s_s[:5]) == list(sw[:5]) == [ss.ROW_NON_FINITE_INPUT, ss.ROW_PENALTY_OVERFLOW, ss.ROW_NO_FINITE_LOGIT,
                                             ss.ROW_TEMPERATURE_OVERFLOW, ss.ROW_OK]
    assert i_s[4] == iw[4]
    assert s_s[5] == ss.ROW_INVALID_ROW and i_s[5] == -1


def test_restrict_slice_with_global_history(engine):
    """ssb_restrict_slice (the restricted-slice exchange's first step, history as the rows' global ids, the
    whole rows' mask) equals the whole rows' restricted logits on the slice's columns, bit for bit."""
    import torch
    c = wl.config4(rows=4)
    x = dev(c["logits_bf16"], torch.bfloat16)
    h = dev(c["history"])
    V = x.shape[1]
    ban = np.zeros((4, V), bool)
    ban[:, ::97] = True
    m = dev(wl.pack_mask(ban).view(np.int32))
    p = ss.params(**c["params"])
    whole = engine.restrict(x, p, h, None, m, ss.MASK_BAN)
    for world in (2, 3, 8):
        for off, width in vs.shard_bounds(V, world):
            out = torch.empty((4, width), dtype=torch.float32, device="cuda")
            engine.restrict_slice(x[:, off:off + width], p, off, V, out, h, m, ss.MASK_BAN)
            torch.cuda.synchronize()
            assert torch.equal(out.view(torch.int32), whole[:, off:off + width].contiguous().view(torch.int32)), (world, off)
