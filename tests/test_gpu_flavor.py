"""The Haru and Drama 3 candidate rules on the device (params.flavor), through the C ABI, against the
compiled reference's golden vectors and the oracle's restatements of haru::candidates
(haru/sampler.cpp:18-61) and drama3::candidates (drama3/sampler.cpp:30-60), each followed by pick().

Tolerances, stated per family:
  * token lists, counts and statuses: identical (integers);
  * Haru's weights (float32 softmax): within (k + 64) 2^-24 absolute, the reference's own allowance for
    another float32 exp and sum (checks/haru/haru-sampling-check.cpp:29-35); the device rounds exp in
    double once to float, glibc's expf is within an ulp of it;
  * Drama 3's weights (exp in double): within 1e-12 relative (CUDA's exp against glibc's, each within an
    ulp);
  * ids: identical, except where u lies within the weight tolerance of a boundary between two
    candidates' cumulative shares (none is expected).
"""
import os

import numpy as np
import pytest

import speech_sampler as ss
import speech_workloads as wl
from oracle import MASK_BAN, MASK_NONE, Oracle, params as oparams
from test_gpu_parity import engine_run

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
HARU, DRAMA3 = ss.FLAVOR_HARU, ss.FLAVOR_DRAMA3
D3_RTOL = 1e-12


def haru_tol(k):
    return (k + 64) * 2.0 ** -24


def load_cases(name):
    z = np.load(os.path.join(GOLDEN, name))
    out = {}
    for key in z.files:
        case, field = key.split("/", 1) if "/" in key else ("", key)
        out.setdefault(case, {})[field] = z[key]
    return out


@pytest.fixture(scope="module")
def orc():
    return Oracle()


def boundary_distance(weights, u):
    """How far u lies from the nearest cumulative share pick() compares it with."""
    w = np.asarray(weights, np.float64)
    if len(w) < 2 or w.sum() == 0:
        return np.inf
    cum = np.cumsum(w / w.sum())[:-1]
    return float(np.min(np.abs(cum - u)))


def family_oracle(orc, flavor, row_f32, t, k, p, u, banned=None):
    """(status, id, tokens, weights) of one restricted row by the family's restatement and pick(). For
    Drama 3, banned columns (-inf after the mask) are removed before the rule and the tokens mapped back:
    the engine's definition of a mask over Drama 3 rows (the reference's rows hold no -inf)."""
    if flavor == HARU:
        st, tok, w = orc.haru_candidates(row_f32, t, k, p)
    else:
        keep = np.nonzero(row_f32 != -np.inf)[0] if banned is not None else np.arange(len(row_f32))
        if len(keep) == 0:
            return 3, -1, np.zeros(0, np.int32), np.zeros(0)
        st, tok, w = orc.drama3_candidates(row_f32[keep], t, k, p)
        tok = keep[tok].astype(np.int32)
    if st != 0:
        return st, -1, tok, w
    return 0, int(tok[orc.pick(w, u)]), tok, w


def check_rows(orc, flavor, x_f32, plist, u, got, banned=None):
    ids, st, tok, w, cnt = got[:5]
    near = 0
    for r in range(x_f32.shape[0]):
        p = plist[r]
        want_st, want_id, want_tok, want_w = family_oracle(orc, flavor, x_f32[r], p.temperature, p.top_k, p.top_p,
                                                           u[r], banned)
        assert st[r] == want_st, (r, st[r], want_st)
        if want_st != 0:
            assert ids[r] == -1
            continue
        n = len(want_tok)
        assert cnt[r] == n, (r, cnt[r], n)
        c = min(n, tok.shape[1])
        assert np.array_equal(tok[r, :c], want_tok[:c]), r
        if flavor == HARU:
            tol = haru_tol(n)
            assert np.max(np.abs(w[r, :c] - want_w[:c]), initial=0) <= tol, r
        else:
            tol = D3_RTOL * float(np.max(want_w))
            assert np.max(np.abs(w[r, :c] - want_w[:c]) / np.maximum(np.abs(want_w[:c]), 1e-300), initial=0) <= D3_RTOL, r
        if ids[r] != want_id:
            assert boundary_distance(want_w, u[r]) <= tol * 4, (r, ids[r], want_id)
            near += 1
    return near


# ---------------------------------------------------------------- the compiled reference's vectors
@pytest.mark.parametrize("case", ["default", "top-p", "greedy", "wide"])
def test_haru_golden_on_device(engine, orc, case):
    g = load_cases("haru_cases.npz")
    x = g[""]["logits"]
    c = g[case]
    p = ss.params(temperature=float(c["t"]), top_k=int(c["k"]), top_p=float(c["p"]), flavor=HARU)
    u = np.random.default_rng(5).random(x.shape[0])
    ids, st, tok, w, cnt, _ = engine_run(engine, x, p, u=u, cap=600)
    assert np.all(st == 0)
    for r in range(x.shape[0]):
        stored = int(c["count"][r])  # the fixture holds at most 600 entries (the full count: check_rows)
        assert cnt[r] == stored if stored < 600 else cnt[r] >= 600
        assert np.array_equal(tok[r, :stored], c["tokens"][r, :stored])
        assert np.max(np.abs(w[r, :stored] - c["weights"][r, :stored])) <= haru_tol(int(cnt[r]))
    check_rows(orc, HARU, x, [p] * x.shape[0], u, (ids, st, tok, w, cnt))


@pytest.mark.parametrize("case", ["card", "main-top-k-1", "codes-top-p-narrow", "codes-cold", "codes-hot",
                                  "main-every-token"])
def test_drama3_golden_on_device(engine, case):
    c = load_cases("drama3_cases.npz")[case]
    x = c["logits"]
    p = ss.params(temperature=float(c["t"]), top_k=int(c["k"]), top_p=float(c["p"]), flavor=DRAMA3)
    cap = c["tokens"].shape[1]
    ids, st, tok, w, cnt, _ = engine_run(engine, x, p, u=c["u"], cap=cap)
    assert np.all(st == 0)
    for r in range(x.shape[0]):
        n = int(c["count"][r])
        assert cnt[r] == n
        assert np.array_equal(tok[r, :n], c["tokens"][r, :n])
        want = c["weights"][r, :n]
        assert np.max(np.abs(w[r, :n] - want) / want) <= D3_RTOL
    assert np.array_equal(ids, c["ids"])
    # the same rows through the product entry point (no export) draw the same ids
    ids2, st2 = engine_run(engine, x, p, u=c["u"])
    assert np.array_equal(ids2, ids) and np.all(st2 == 0)


# ---------------------------------------------------------------- random rows against the oracle
def _random_family_batch(rng, flavor, n, rows, dtype):
    scale = float(rng.choice([0.5, 2.0, 6.0]))
    x = (rng.standard_normal((rows, n)) * scale).astype(np.float32)
    if rng.random() < 0.3:
        x = np.round(x).astype(np.float32)  # ties
    if flavor == HARU and rng.random() < 0.4:
        x[:, rng.choice(n, max(1, n // 20), replace=False)] = -np.inf  # the session's bans
    if dtype == "bf16":
        bits = wl.to_bf16_bits(x)
        return bits, wl.bf16_bits_to_f32(bits)
    return x, x


@pytest.mark.parametrize("flavor", [HARU, DRAMA3])
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_family_random_rows(engine, orc, flavor, dtype):
    rng = np.random.default_rng(100 + flavor * 10 + (dtype == "bf16"))
    for trial in range(10):
        n = int(rng.choice([5, 300, 4096, 4097, 9000, 32000, 151936]))
        rows = int(rng.choice([1, 3, 16]))
        t = float(rng.choice([0.0, 1e-6, 0.6, 1.0, 1.7]))
        k = int(rng.choice([1, 30, 100, 500, 4097])) if n > 8192 else int(rng.choice([0, 1, 30, 500, n, n + 3]))
        if flavor == HARU and n > 8192 and t > 0 and k == 0:
            k = 50
        p = ss.params(temperature=t, top_k=k, top_p=float(rng.choice([0.0, 0.1, 0.9, 1.0])), flavor=flavor)
        x, xf = _random_family_batch(rng, flavor, n, rows, dtype)
        u = rng.random(rows)
        kk = k if k > 0 else (n if flavor == HARU else 1)
        got = engine_run(engine, x, p, u=u, cap=min(kk, n, 8192))
        check_rows(orc, flavor, xf, [p] * rows, u, got)


@pytest.mark.parametrize("flavor", [HARU, DRAMA3])
def test_family_penalties_and_mask(engine, orc, flavor):
    """The engine's logit processors before the family's rule: repetition/presence/frequency penalties
    over the history and a ban mask, restricted by the oracle's restricted() and handed to the family's
    restatement."""
    rng = np.random.default_rng(31 + flavor)
    for n, rows in ((4096, 8), (4097, 4), (151936, 3)):
        x = (rng.standard_normal((rows, n)) * 2.0).astype(np.float32)
        hist = rng.integers(-3, n + 3, size=(rows, 200)).astype(np.int32)
        hist[:, :40] = np.argsort(-x, axis=1)[:, :40]  # the best tokens repeat
        ban = rng.random((rows, n)) < 0.05
        mask = wl.pack_mask(ban)
        p = ss.params(temperature=0.8, top_k=50, top_p=0.9, repetition_penalty=1.3, presence_penalty=0.2,
                      frequency_penalty=0.05, flavor=flavor)
        op = oparams(greedy=True, repetition_penalty=1.3, presence_penalty=0.2, frequency_penalty=0.05)
        u = rng.random(rows)
        got = engine_run(engine, x, p, history=hist, mask=mask, mask_kind=MASK_BAN, u=u, cap=50)
        restricted = np.stack([orc.sample_row(x[r], op, hist[r], mask[r], MASK_BAN, want_processed=True)["processed"]
                               for r in range(rows)])
        assert np.array_equal(got[5], restricted)
        check_rows(orc, flavor, restricted, [p] * rows, u, got, banned=ban)


# ---------------------------------------------------------------- refusals and edges
def test_family_refusals(engine):
    n = 4097
    base = np.linspace(-4, 4, n).astype(np.float32)
    u = np.full(1, 0.5)
    for flavor in (HARU, DRAMA3):
        p = ss.params(temperature=0.9, top_k=30, top_p=0.9, flavor=flavor)
        for bad in (np.nan, np.inf):
            y = base.copy()[None]
            y[0, 11] = bad
            assert engine_run(engine, y, p, u=u)[1][0] == ss.ROW_NON_FINITE_INPUT
    # -inf is a ban for Haru, a device fault for Drama 3
    y = base.copy()[None]
    y[0, 5] = -np.inf
    ids, st = engine_run(engine, y, ss.params(temperature=0.9, top_k=30, flavor=HARU), u=u)
    assert st[0] == 0
    assert engine_run(engine, y, ss.params(temperature=0.9, top_k=30, flavor=DRAMA3), u=u)[1][0] == \
        ss.ROW_NON_FINITE_INPUT
    # a temperature that scales a finite logit beyond a float
    big = (base * np.float32(1e34))[None]
    assert engine_run(engine, big, ss.params(temperature=1e-38, top_k=30, flavor=HARU), u=u)[1][0] == \
        ss.ROW_TEMPERATURE_OVERFLOW
    assert engine_run(engine, big, ss.params(temperature=0.0, top_k=30, flavor=DRAMA3), u=u)[1][0] == \
        ss.ROW_TEMPERATURE_OVERFLOW
    # Haru at T <= 0: the first maximum, no draw (u not needed); Drama 3 with top_k 0 keeps one token
    z = np.zeros((1, n), np.float32)
    z[0, [17, 40]] = 3.0
    ids, st = engine_run(engine, z, ss.params(temperature=0.0, flavor=HARU))
    assert st[0] == 0 and ids[0] == 17
    ids, st = engine_run(engine, z, ss.params(temperature=1.0, top_k=0, flavor=DRAMA3), u=np.full(1, 0.99))
    assert st[0] == 0 and ids[0] == 17
    # more candidates than the kernel holds: refused on the host
    wide = np.zeros((1, 20000), np.float32)
    with pytest.raises(ss.SsbError) as e:
        engine_run(engine, wide, ss.params(temperature=1.0, top_k=0, flavor=HARU), u=u)
    assert e.value.status == ss.OUT_OF_RANGE
    # every token banned over Drama 3 rows
    ban = wl.pack_mask(np.ones((1, n), bool))
    ids, st = engine_run(engine, base[None], ss.params(temperature=1.0, top_k=5, flavor=DRAMA3), mask=ban,
                         mask_kind=MASK_BAN, u=u)
    assert st[0] == ss.ROW_NO_FINITE_LOGIT and ids[0] == -1


def test_family_row_params(engine, orc):
    """Per-row settings: rows of the call's family follow their own settings; a row of another family,
    or one keeping more candidates than the launch's bound (max_top_k), is INVALID_ROW."""
    rng = np.random.default_rng(8)
    n, rows = 4096, 6
    x = (rng.standard_normal((rows, n)) * 3).astype(np.float32)
    plist = [ss.params(temperature=0.7, top_k=25, top_p=1.0, flavor=HARU),
             ss.params(temperature=1.5, top_k=100, top_p=0.95, flavor=HARU),
             ss.params(temperature=0.0, top_k=25, flavor=HARU),
             ss.params(temperature=0.9, top_k=30, flavor=DRAMA3),
             ss.params(temperature=0.9, top_k=30),
             ss.params(temperature=0.9, top_k=400, flavor=HARU)]
    u = rng.random(rows)
    ids, st, tok, w, cnt, _ = engine_run(engine, x, plist[0], u=u, row_params=plist, max_top_k=128, cap=128)
    assert list(st[3:]) == [ss.ROW_INVALID_ROW] * 3 and np.all(ids[3:] == -1)
    check_rows(orc, HARU, x[:3], plist[:3], u[:3], (ids[:3], st[:3], tok[:3], w[:3], cnt[:3]))
