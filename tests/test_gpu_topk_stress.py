"""The large-vocabulary path for top-k <= 128 on aligned rows (the top-k kernel, ssb_topk.cu) against
the oracle restatement, on rows built to stress a streamed top-k: ascending rows (every block a new
maximum, so a bound from part of the row is poor) and descending ones (the first blocks hold the
best), the best tokens all penalized history tokens or banned, fewer allowed tokens than k, NaN and
infinities, ragged tails behind aligned rows, one row split over many CTAs and whole rows per CTA. Token ids and
statuses must equal the oracle's (a draw within 1e-12 of a cumulative-share boundary would be allowed
and counted; none is expected)."""
import numpy as np
import pytest

import speech_sampler as ss
import speech_workloads as wl
from oracle import MASK_ALLOW, MASK_BAN, MASK_NONE, params
from test_gpu_parity import assert_ids, engine_run

pytestmark = pytest.mark.gpu


def _check(engine, oracle, x, kw, hist=None, hlen=None, mask=None, kind=MASK_NONE, u=None, ld=None):
    op = params(**kw)
    rows = x.shape[0]
    u = np.zeros(rows) if u is None else u
    want_ids, want_st = [], []
    for r in range(rows):
        h = None if hist is None else (hist[r] if hlen is None else hist[r, :hlen[r]])
        o = oracle.sample_row(x[r], op, h, None if mask is None else (mask if mask.ndim == 1 else mask[r]), kind, u[r])
        want_ids.append(o["id"])
        want_st.append(o["status"])
    ids, st = engine_run(engine, x, ss.params(**kw), hist, hlen, mask, kind, u, ld=ld)
    near = assert_ids(oracle, ids, st, np.array(want_ids), np.array(want_st), x, lambda r: op,
                      lambda r: None if hist is None else (hist[r] if hlen is None else hist[r, :hlen[r]]),
                      lambda r: None if mask is None else (mask if mask.ndim == 1 else mask[r]), kind, u)
    assert near == 0
    return ids, st


@pytest.mark.parametrize("bf16", [False, True])
@pytest.mark.parametrize("rows", [1, 8, 64])
@pytest.mark.parametrize("kw", [dict(greedy=True), dict(temperature=0.8, top_k=40, top_p=0.95),
                                dict(temperature=1.3, top_k=128, top_p=0.9)])
def test_ascending_rows_cut_the_buffers(engine, oracle, bf16, rows, kw):
    """Rising logits: the first blocks hold the smallest, so any bound taken early lets nearly everything
    through."""
    v = 151936
    rng = np.random.default_rng(rows * 7 + bf16)
    x = (np.linspace(-8.0, 8.0, v, dtype=np.float32)[None, :] + rng.standard_normal((rows, v)).astype(np.float32) * 0.01)
    x = wl.to_bf16_bits(x) if bf16 else x
    u = rng.random(rows, dtype=np.float32).astype(np.float64)
    _check(engine, oracle, x, kw, u=u)


@pytest.mark.parametrize("rows", [1, 16])
def test_descending_rows(engine, oracle, rows):
    v = 151936
    rng = np.random.default_rng(rows)
    x = np.linspace(8.0, -8.0, v, dtype=np.float32)[None, :] + rng.standard_normal((rows, v)).astype(np.float32) * 0.01
    u = rng.random(rows, dtype=np.float32).astype(np.float64)
    _check(engine, oracle, x, dict(temperature=0.9, top_k=50, top_p=0.9), u=u)
    _check(engine, oracle, x, dict(greedy=True))


@pytest.mark.parametrize("rows", [2, 40])
def test_best_tokens_are_history_or_banned(engine, oracle, rows):
    """The 300 largest logits of each row are history tokens with a heavy penalty, or banned: the raw
    block maxima overstate every restricted logit there, and the penalized values decide."""
    v = 151936
    rng = np.random.default_rng(11 + rows)
    x = rng.standard_normal((rows, v)).astype(np.float32)
    top = np.argsort(-x, axis=1)[:, :300]
    hist = np.concatenate([top, top[:, :100]], axis=1).astype(np.int32)  # 100 of them twice
    kw = dict(temperature=0.8, top_k=40, top_p=0.95, repetition_penalty=3.0, presence_penalty=2.0,
              frequency_penalty=0.5)
    u = rng.random(rows, dtype=np.float32).astype(np.float64)
    _check(engine, oracle, x, kw, hist=hist, u=u)
    _check(engine, oracle, x, dict(greedy=True, repetition_penalty=3.0), hist=hist)
    ban = np.zeros((rows, v), bool)
    np.put_along_axis(ban, top, True, axis=1)
    _check(engine, oracle, x, dict(temperature=0.8, top_k=40, top_p=0.95), mask=wl.pack_mask(ban), kind=MASK_BAN, u=u)
    _check(engine, oracle, x, dict(greedy=True), mask=wl.pack_mask(ban), kind=MASK_BAN)


def test_fewer_allowed_than_k(engine, oracle):
    """An allow mask with 30 tokens and top-k 100: the candidates include -inf tokens."""
    v, rows = 151936, 3
    rng = np.random.default_rng(5)
    x = rng.standard_normal((rows, v)).astype(np.float32)
    allow = np.zeros((rows, v), bool)
    for r in range(rows):
        allow[r, rng.choice(v, 30, replace=False)] = True
    u = rng.random(rows, dtype=np.float32).astype(np.float64)
    _check(engine, oracle, x, dict(temperature=1.0, top_k=100, top_p=1.0), mask=wl.pack_mask(allow), kind=MASK_ALLOW,
           u=u)
    _check(engine, oracle, x, dict(greedy=True), mask=wl.pack_mask(allow), kind=MASK_ALLOW)


@pytest.mark.parametrize("bf16", [False, True])
def test_nonfinite_values(engine, oracle, bf16):
    v, rows = 151936, 6
    rng = np.random.default_rng(3)
    x = rng.standard_normal((rows, v)).astype(np.float32)
    hist = rng.integers(0, v, size=(rows, 64)).astype(np.int32)
    x[0, 1000] = np.nan                      # NaN -> NON_FINITE_INPUT
    x[1, hist[1, 3]] = np.nan                # NaN at a history token -> NON_FINITE_INPUT
    x[2, 77] = np.inf                        # +inf with a penalty -> PENALTY_OVERFLOW
    x[3, 5:20000] = -np.inf                  # many -inf, the rest finite
    x[4, 150000] = np.inf                    # +inf, no penalty on the row -> NO_FINITE_LOGIT
    ban = np.zeros((rows, v), bool)
    ban[5, 123] = True
    x[5, 123] = np.nan                       # NaN under the ban -> fine
    xx = wl.to_bf16_bits(x) if bf16 else x
    u = np.full(rows, 0.4)
    kw = dict(temperature=0.9, top_k=30, repetition_penalty=1.1)
    _check(engine, oracle, xx[:4], kw, hist=hist[:4], u=u[:4])
    _check(engine, oracle, xx[4:5], dict(temperature=0.9, top_k=30), u=u[4:5])
    _check(engine, oracle, xx[5:6], kw, hist=hist[5:6], mask=wl.pack_mask(ban[5:6]), kind=MASK_BAN, u=u[5:6])


@pytest.mark.parametrize("vocab", [151939, 9001, 200003])
@pytest.mark.parametrize("bf16", [False, True])
def test_ragged_tails_on_aligned_rows(engine, oracle, vocab, bf16):
    """Rows whose length is not a whole number of 16-byte groups, at a 16-byte-aligned pitch: the last
    columns are taken outside the stream."""
    rows = 5
    rng = np.random.default_rng(vocab + bf16)
    x = (rng.standard_normal((rows, vocab)) * 2).astype(np.float32)
    x[:, -1] = 9.0  # the best token in the tail
    x = wl.to_bf16_bits(x) if bf16 else x
    es = 2 if bf16 else 4
    ld = -(-vocab * es // 16) * 16 // es
    u = rng.random(rows, dtype=np.float32).astype(np.float64)
    _check(engine, oracle, x, dict(temperature=0.7, top_k=20, top_p=0.9), u=u, ld=ld)
    _check(engine, oracle, x, dict(greedy=True), ld=ld)


@pytest.mark.parametrize("rows", [1, 3, 37, 300])
def test_random_settings_large_vocab(engine, oracle, rows):
    """Random settings over the top-k kernel's range (top-k <= 128, aligned rows), penalties, masks."""
    rng = np.random.default_rng(rows)
    v = int(rng.choice([9000, 65536, 151936]))
    x = (rng.standard_normal((rows, v)) * rng.choice([1.0, 3.0])).astype(np.float32)
    bf16 = rows % 2 == 1
    xx = wl.to_bf16_bits(x) if bf16 else x
    plist = []
    for r in range(rows):
        plist.append(dict(greedy=bool(rng.random() < 0.2), temperature=float(rng.choice([0.5, 0.8, 1.0, 1.7])),
                          top_k=int(rng.choice([1, 2, 40, 50, 128])), top_p=float(rng.choice([1.0, 0.95, 0.5])),
                          repetition_penalty=float(rng.choice([1.0, 1.05])), presence_penalty=float(rng.choice([0.0, 0.5])),
                          frequency_penalty=float(rng.choice([0.0, 0.3]))))
    hist = rng.integers(-2, v + 2, size=(rows, 200)).astype(np.int32)
    ban = wl.pack_mask(rng.random((rows, v)) < 0.02)
    u = rng.random(rows, dtype=np.float32).astype(np.float64)
    want = [oracle.sample_row(xx[r], params(**plist[r]), hist[r], ban[r], MASK_BAN, u[r]) for r in range(rows)]
    ids, st = engine_run(engine, xx, ss.params(), hist, None, ban, MASK_BAN, u,
                         row_params=[ss.params(**q) for q in plist], max_top_k=128)
    assert np.array_equal(st, [w["status"] for w in want])
    assert np.array_equal(ids, [w["id"] for w in want])
