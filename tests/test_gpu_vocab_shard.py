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
