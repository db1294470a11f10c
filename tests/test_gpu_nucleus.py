"""Parity of the large-vocabulary kernel for rows that keep more than 1024 tokens (top-k 0 = every
token: the constrained-decoding sweep, configuration 5) with the oracle: token ids exactly equal (a
mismatch is tolerated only within 1e-12 of a cumulative-share boundary, as in test_gpu_parity), statuses
exactly equal. The fast path (histogram of the softmax mass, the two crossing buckets sorted) and the
exact path (every kept token sorted, the reference's sequential sums) are both exercised: the candidate
export always takes the exact path, and so do rows whose top_p no running share reaches."""
import numpy as np
import pytest

import speech_sampler as ss
import speech_workloads as wl
from oracle import MASK_ALLOW, MASK_BAN, MASK_NONE, params

from test_gpu_parity import assert_ids, engine_run

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("density", [0.001, 0.01, 0.1, 0.5])
def test_config5_allow_mask(engine, oracle, density):
    c = wl.config5(rows=6, density=density)
    p = params(**c["params"])
    ids, st = engine_run(engine, c["logits"], ss.params(**c["params"]), mask=c["mask"], mask_kind=MASK_ALLOW, u=c["u"])
    want, wst, _ = oracle.sample_rows(c["logits"], p, mask=c["mask"], mask_kind=MASK_ALLOW, u=c["u"])
    near = assert_ids(oracle, ids, st, want, wst, c["logits"], lambda r: p, lambda r: None, lambda r: c["mask"][r],
                      MASK_ALLOW, c["u"])
    assert near == 0


def test_every_token_no_mask(engine, oracle):
    rng = np.random.default_rng(51)
    x = (rng.standard_normal((4, 151936), dtype=np.float32) * np.float32(2.0))
    u = rng.random(4)
    for kw in (dict(temperature=1.0, top_k=0, top_p=0.9), dict(temperature=0.7, top_k=0, top_p=0.5),
               dict(temperature=1.3, top_k=5000, top_p=0.95)):
        p = params(**kw)
        ids, st = engine_run(engine, x, ss.params(**kw), u=u)
        want, wst, _ = oracle.sample_rows(x, p, u=u)
        assert_ids(oracle, ids, st, want, wst, x, lambda r: p, lambda r: None, lambda r: None, MASK_NONE, u)


@pytest.mark.parametrize("scale,kw", [
    (30.0, dict(temperature=1.0, top_k=0, top_p=0.9)),      # most tokens 64 or more below the maximum
    (30.0, dict(temperature=1.0, top_k=0, top_p=0.999)),
    (2.0, dict(temperature=0.05, top_k=0, top_p=0.9)),      # a small temperature: the same spread, scaled
    (0.01, dict(temperature=1.0, top_k=0, top_p=0.9)),      # nearly flat: the mass in a handful of buckets
])
def test_mass_spread(engine, oracle, scale, kw):
    """The mass histogram's buckets are 1/64 wide below the row's maximum scaled logit, and every token
    64 or more below shares the lowest: rows far wider and far narrower than that."""
    rng = np.random.default_rng(int(scale * 100) + int(kw["top_p"] * 1000))
    x = (rng.standard_normal((4, 151936), dtype=np.float32) * np.float32(scale))
    allow = rng.random((4, 151936)) < 0.5
    mask = wl.pack_mask(allow)
    u = rng.random(4)
    p = params(**kw)
    ids, st = engine_run(engine, x, ss.params(**kw), mask=mask, mask_kind=MASK_ALLOW, u=u)
    want, wst, _ = oracle.sample_rows(x, p, mask=mask, mask_kind=MASK_ALLOW, u=u)
    near = assert_ids(oracle, ids, st, want, wst, x, lambda r: p, lambda r: None, lambda r: mask[r], MASK_ALLOW, u)
    assert near == 0


def test_bf16_history_large_k(engine, oracle):
    c = wl.config4(rows=4)
    kw = dict(c["params"], top_k=2000)
    p = params(**kw)
    ids, st = engine_run(engine, c["logits_bf16"], ss.params(**kw), c["history"], u=c["u"])
    want, wst, _ = oracle.sample_rows(c["logits_bf16"], p, history=c["history"], u=c["u"])
    assert_ids(oracle, ids, st, want, wst, c["logits_bf16"], lambda r: p, lambda r: c["history"][r], lambda r: None,
               MASK_NONE, c["u"])


def test_no_cut_and_single_token(engine, oracle):
    """top_p 1: every token (the -inf ones too) is kept and pick()'s fallback is the last of them; an
    allow mask of one token; a ban mask over everything but three tokens."""
    rng = np.random.default_rng(52)
    v = 20000
    x = rng.standard_normal((3, v), dtype=np.float32)
    allow = np.zeros((3, v), bool)
    allow[0, rng.choice(v, 300, replace=False)] = True
    allow[1, 777] = True
    allow[2, [5, 6000, 19999]] = True
    m = wl.pack_mask(allow)
    for kw, u in ((dict(top_k=0, top_p=1.0), np.array([0.3, 0.99, 0.999999])),
                  (dict(top_k=0, top_p=0.9), np.array([0.0, 0.5, 1.0]))):
        p = params(**kw)
        ids, st = engine_run(engine, x, ss.params(**kw), mask=m, mask_kind=MASK_ALLOW, u=u)
        want, wst, _ = oracle.sample_rows(x, p, mask=m, mask_kind=MASK_ALLOW, u=u)
        assert_ids(oracle, ids, st, want, wst, x, lambda r: p, lambda r: None, lambda r: m[r], MASK_ALLOW, u)


def test_candidates_export_exact_path(engine, oracle):
    c = wl.config5(rows=3, density=0.01)
    p = params(**c["params"])
    cap = 64
    ids, st, tok, w, cnt, _ = engine_run(engine, c["logits"], ss.params(**c["params"]), mask=c["mask"],
                                         mask_kind=MASK_ALLOW, u=c["u"], cap=cap)
    for r in range(3):
        o = oracle.sample_row(c["logits"][r], p, None, c["mask"][r], MASK_ALLOW, c["u"][r], cap=cap)
        assert ids[r] == o["id"] and st[r] == o["status"] == ss.ROW_OK
        assert cnt[r] == o["count"]
        m = min(cap, o["count"])
        assert np.array_equal(tok[r, :m], o["tokens"][:m])
        np.testing.assert_allclose(w[r, :m], o["weights"][:m], rtol=1e-12, atol=0)


def test_statuses_and_mixed_rows(engine, oracle):
    """NaN and all-banned rows, a greedy row and per-row top-k in one launch (max_top_k 0)."""
    rng = np.random.default_rng(53)
    v = 30000
    x = rng.standard_normal((4, v), dtype=np.float32)
    x[1, 123] = np.nan
    ban = np.zeros((4, v), bool)
    ban[2] = True
    m = wl.pack_mask(ban)
    rows = [params(top_k=0, top_p=0.9), params(top_k=0, top_p=0.9), params(top_k=0, top_p=0.9), params(greedy=True)]
    u = rng.random(4)
    ids, st = engine_run(engine, x, ss.params(top_k=0, top_p=0.9), mask=m, mask_kind=MASK_BAN, u=u,
                         row_params=[ss.params(greedy=bool(r.greedy), top_k=r.top_k, top_p=r.top_p) for r in rows],
                         max_top_k=0)
    want, wst, _ = oracle.sample_rows(x, rows, mask=m, mask_kind=MASK_BAN, u=u)
    assert list(st) == list(wst)
    assert list(ids) == list(want)


def test_reserve_then_graph_capture(oracle):
    """ssb_context_reserve sizes the nucleus lists, so a top-k 0 launch can be captured into a CUDA graph
    by a fresh context (capture forbids cudaMalloc) and replayed."""
    import torch
    c = wl.config5(rows=8, density=0.01)
    p = params(**c["params"])
    s = ss.Sampler(0)
    try:
        s.reserve(8, 151936)
        x = torch.from_numpy(c["logits"]).cuda()
        m = torch.from_numpy(c["mask"].view(np.int32)).cuda()
        u = torch.from_numpy(c["u"]).cuda()
        ids = torch.empty(8, dtype=torch.int32, device="cuda")
        st = torch.empty(8, dtype=torch.int32, device="cuda")
        stream = torch.cuda.Stream()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            s.sample(x, ss.params(**c["params"]), mask=m, mask_kind=MASK_ALLOW, u=u, ids=ids, status=st,
                     stream=torch.cuda.current_stream())
        ids.fill_(-7)
        g.replay()
        torch.cuda.synchronize()
        want, wst, _ = oracle.sample_rows(c["logits"], p, mask=c["mask"], mask_kind=MASK_ALLOW, u=c["u"])
        assert list(st.cpu().numpy()) == list(wst)
        assert list(ids.cpu().numpy()) == list(want)
        del g
    finally:
        s.close()


@pytest.mark.parametrize("density", [0.001, 0.5])
def test_config5_batch_4096(engine, oracle, density):
    """Configuration 5 at its largest batch, B = 4096 rows of 151936 tokens (2.5 GB of fp32 logits): more
    rows than the grid holds CTAs, so every CTA loops over rows and reuses its candidate-list region. 64
    rows spread over the batch (the first and last, and rows past each multiple of the grid) are checked
    against the oracle; every status must be OK."""
    c = wl.config5(rows=4096, density=density)
    p = params(**c["params"])
    ids, st = engine_run(engine, c["logits"], ss.params(**c["params"]), mask=c["mask"], mask_kind=MASK_ALLOW, u=c["u"])
    assert np.all(st == ss.ROW_OK)
    rng = np.random.default_rng(7)
    pick = np.unique(np.concatenate([[0, 1, 147, 148, 149, 295, 296, 297, 1023, 2048, 4094, 4095],
                                     rng.choice(4096, 52, replace=False)]))[:64]
    want, wst, _ = oracle.sample_rows(c["logits"][pick], p, mask=c["mask"][pick], mask_kind=MASK_ALLOW,
                                      u=c["u"][pick])
    near = assert_ids(oracle, ids[pick], st[pick], want, wst, c["logits"][pick], lambda r: p, lambda r: None,
                      lambda r: c["mask"][pick][r], MASK_ALLOW, c["u"][pick])
    assert near == 0


@pytest.mark.parametrize("density", [0.001, 0.01, 0.1, 0.5])
def test_config5_batch_1(engine, oracle, density):
    """Configuration 5 at B = 1: one-row calls (one CTA for the whole row), 16 rows per density, each
    against the oracle."""
    c = wl.config5(rows=16, density=density, row0=5000)
    p = params(**c["params"])
    for r in range(16):
        ids, st = engine_run(engine, c["logits"][r:r + 1], ss.params(**c["params"]), mask=c["mask"][r:r + 1],
                             mask_kind=MASK_ALLOW, u=c["u"][r:r + 1])
        o = oracle.sample_row(c["logits"][r], p, None, c["mask"][r], MASK_ALLOW, c["u"][r])
        assert st[0] == o["status"] == ss.ROW_OK and ids[0] == o["id"], (r, ids[0], o["id"])
