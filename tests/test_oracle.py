"""The oracle restatement (oracle/sampler_oracle.c), pinned against the reference's own sampler:
golden fixtures the compiled reference produced (tests/golden/make_golden.py), the known answers of
the reference's checks, and — where the reference is built here — randomized agreement with it.
CPU only."""
import json
import os

import numpy as np
import pytest

import speech_workloads as wl
from oracle import MASK_ALLOW, MASK_BAN, params

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load_cases(name):
    z = np.load(os.path.join(GOLDEN, name))
    cases = {}
    for key in z.files:
        if "/" not in key:
            cases.setdefault("", {})[key] = z[key]
            continue
        case, field = key.split("/", 1)
        cases.setdefault(case, {})[field] = z[key]
    return cases


# ---------------------------------------------------------------- known answers
def test_pick_edges_match_reference_check(oracle):
    """checks/qwen3-tts/qwen3-tts-sampler-check.cpp:98-102: a draw equal to a share passes to the next."""
    k = json.load(open(os.path.join(GOLDEN, "kat.json")))
    for e, want in zip(k["pick_edges"], k["pick_results"]):
        assert oracle.pick(k["pick_weights"], e) == want
    assert oracle.pick([5.0], 1.0) == k["pick_single"] == 0
    assert k["pick_results"] == [0, 0, 1, 1, 2, 3, 3]


def test_uniform_stream_bit_exact(oracle):
    """uniform() over std::mt19937_64(1) (sampling.cpp:5-7), bit for bit, and the shares of 400,000
    draws picked from weights 1, 2, 3, 4 within 0.004 (qwen3-tts-sampler-check.cpp:103-113)."""
    k = json.load(open(os.path.join(GOLDEN, "kat.json")))
    draws = oracle.uniform(1, 400000)
    assert [float(x).hex() for x in draws[:16]] == k["uniform_seed1_first16"]
    assert np.all((draws >= 0) & (draws <= 1))
    # pick() = first cumulative share > u; the shares 1/10, 2/10, 3/10 accumulate in order
    cum = np.cumsum(np.array([1.0, 2.0, 3.0]) / 10.0)
    picks = np.searchsorted(cum, draws, side="right")
    for u in draws[:2000]:
        assert oracle.pick([1.0, 2.0, 3.0, 4.0], u) == np.searchsorted(cum, u, side="right")
    shares = np.bincount(picks, minlength=4) / len(draws)
    assert np.array_equal(shares, np.array(k["uniform_seed1_shares"]))
    assert np.max(np.abs(shares - [0.1, 0.2, 0.3, 0.4])) <= 0.004


def test_penalty_overflow_refused(oracle):
    """A penalty of 1e-40 on logits 1, 2 both in the history: refused by greedy and by a draw
    (qwen3-tts-sampler-check.cpp:70-91), status PENALTY_OVERFLOW = the Error naming repetition_penalty."""
    k = json.load(open(os.path.join(GOLDEN, "kat.json")))
    for greedy, want in zip((True, False), k["penalty_1e-40_status"]):
        r = oracle.sample_row(np.array([1.0, 2.0], np.float32), params(greedy=greedy, repetition_penalty=1e-40),
                              np.array([0, 1], np.int32), u=0.5)
        assert r["status"] == want == 1


def test_temperature_overflow_refused(oracle):
    """Temperature 1e-38 takes a logit beyond a float: TEMPERATURE_OVERFLOW (graph-sampler-check.cpp:163-186)."""
    k = json.load(open(os.path.join(GOLDEN, "kat.json")))
    row = np.random.default_rng(k["temperature_1e-38_row_seed"]).standard_normal(2048, dtype=np.float32) * np.float32(1.5)
    r = oracle.sample_row(row, params(temperature=1e-38, top_k=50), u=0.5)
    assert r["status"] == k["temperature_1e-38_status"] == 2


# ---------------------------------------------------------------- golden cases of the reference
@pytest.mark.parametrize("case", sorted(load_cases("qwen3_tts_cases.npz")))
def test_qwen3_tts_case(oracle, case):
    c = load_cases("qwen3_tts_cases.npz")[case]
    settings = json.loads(str(c["settings"]))
    stack = settings.pop("stack")
    p = params(**settings)
    vocab = c["logits"].shape[1]
    for r in range(c["logits"].shape[0]):
        h = c["history"][r][c["history"][r] >= 0]
        mask = wl.pack_mask(c["banned"][r]) if stack == "talker" else None
        for j in range(c["u"].shape[1]):
            res = oracle.sample_row(c["logits"][r], p, h, mask, MASK_BAN, c["u"][r, j], cap=vocab)
            assert res["status"] == c["status"][r, j]
            assert res["id"] == c["ids"][r, j], (case, r, j)
        if not p.greedy:
            n = int(c["cand_count"][r])
            assert res["count"] == n
            m = min(n, c["cand_tokens"].shape[1])
            w_ref, t_ref = c["cand_weights"][r, :m], c["cand_tokens"][r, :m]
            # identical where the weight is positive (the reference orders tied -inf tokens arbitrarily)
            pos = w_ref > 0
            assert np.array_equal(res["tokens"][:m][pos], t_ref[pos])
            assert np.array_equal(res["weights"][:m], w_ref)


def test_large_vocab_golden(oracle):
    g = load_cases("large_vocab_cases.npz")
    c1 = wl.config1(rows=int(g["config1"]["rows"]))
    ids, status, _ = oracle.sample_rows(c1["logits"], params(greedy=True), mask=c1["mask"], mask_kind=MASK_BAN)
    assert np.array_equal(ids, g["config1"]["ids"]) and np.all(status == 0)
    c4 = wl.config4(rows=int(g["config4_rep"]["rows"]))
    p4 = params(temperature=0.8, top_k=40, top_p=0.95, repetition_penalty=1.1)
    x = wl.bf16_bits_to_f32(c4["logits_bf16"])
    ids, status, _ = oracle.sample_rows(x, p4, history=c4["history"], u=c4["u"])
    assert np.array_equal(ids, g["config4_rep"]["ids"])
    # the same rows given as bf16 bits widen to the same fp32 values
    ids2, _, _ = oracle.sample_rows(c4["logits_bf16"], p4, history=c4["history"], u=c4["u"])
    assert np.array_equal(ids2, ids)
    c5 = wl.config5(rows=int(g["config5_d0.01"]["rows"]), density=float(g["config5_d0.01"]["density"]))
    ids, status, _ = oracle.sample_rows(c5["logits"], params(temperature=1.0, top_k=0, top_p=0.9), mask=c5["mask"],
                                        mask_kind=MASK_ALLOW, u=c5["u"])
    assert np.array_equal(ids, g["config5_d0.01"]["ids"])


@pytest.mark.parametrize("case", ["default", "top-p", "greedy", "wide"])
def test_haru_golden(oracle, case):
    g = load_cases("haru_cases.npz")
    x = g[""]["logits"]
    c = g[case]
    for r in range(x.shape[0]):
        st, tok, w = oracle.haru_candidates(x[r], float(c["t"]), int(c["k"]), float(c["p"]), cap=600)
        n = int(c["count"][r])
        assert st == 0 and len(tok) == min(n, 600)
        assert np.array_equal(tok, c["tokens"][r, :len(tok)])
        assert np.array_equal(w, c["weights"][r, :len(tok)])


@pytest.mark.parametrize("case", ["card", "main-top-k-1", "codes-top-p-narrow", "codes-cold", "codes-hot",
                                  "main-every-token"])
def test_drama3_golden(oracle, case):
    """drama3::candidates() (drama3/sampler.cpp:30-60) as the compiled reference returned it: tokens and
    weights bit for bit, and the id pick() draws from them."""
    c = load_cases("drama3_cases.npz")[case]
    for r in range(c["logits"].shape[0]):
        st, tok, w = oracle.drama3_candidates(c["logits"][r], float(c["t"]), int(c["k"]), float(c["p"]))
        n = int(c["count"][r])
        assert st == 0 and len(tok) == n
        assert np.array_equal(tok, c["tokens"][r, :n])
        assert np.array_equal(w, c["weights"][r, :n])
        assert tok[oracle.pick(w, c["u"][r])] == c["ids"][r]


def test_drama3_refusals(oracle):
    """Any non-finite logit is the device's error (status 4, drama3/sampler.cpp:35-37); a temperature
    that takes the largest logit beyond a float overflows (2, :46-47); a temperature under 1e-5 divides
    by 1e-5 (:31); top_k below 1 keeps one token (:40)."""
    x = np.linspace(-3, 3, 300).astype(np.float32)
    for bad in (np.nan, np.inf, -np.inf):
        y = x.copy()
        y[7] = bad
        assert oracle.drama3_candidates(y, 1.0, 30, 0.9)[0] == 4
    big = x * np.float32(1e34)
    assert oracle.drama3_candidates(big, 1e-5, 30, 0.9)[0] == 2
    a = oracle.drama3_candidates(x, 0.0, 30, 1.0)
    b = oracle.drama3_candidates(x, 1e-5, 30, 1.0)
    assert a[0] == 0 and np.array_equal(a[1], b[1]) and np.array_equal(a[2], b[2])
    st, tok, w = oracle.drama3_candidates(x, 1.0, 0, 1.0)
    assert st == 0 and list(tok) == [299] and list(w) == [1.0]


# ---------------------------------------------------------------- extensions (parity unpinned)
def test_presence_frequency_definition(oracle):
    """l -= frequency * count; l -= presence, after the repetition penalty, once per distinct id."""
    x = np.array([2.0, -1.0, 0.5, 3.0], np.float32)
    h = np.array([0, 0, 0, 1, 7, -1], np.int32)  # 7 and -1 are out of range: skipped
    p = params(greedy=True, repetition_penalty=1.25, presence_penalty=0.5, frequency_penalty=0.3)
    r = oracle.sample_row(x, p, h, want_processed=True)
    f = np.float32
    want0 = f(f(f(f(2.0) / f(1.25)) - f(f(0.3) * f(3))) - f(0.5))
    want1 = f(f(f(f(-1.0) * f(1.25)) - f(f(0.3) * f(1))) - f(0.5))
    assert r["processed"][0] == want0 and r["processed"][1] == want1
    assert r["processed"][2] == f(0.5) and r["processed"][3] == f(3.0)
    assert r["id"] == 3


def test_allow_mask_is_complement_of_ban(oracle):
    rng = np.random.default_rng(0)
    x = rng.standard_normal(5000).astype(np.float32)
    allow = rng.random(5000) < 0.1
    p = params(temperature=0.7, top_k=20, top_p=0.9)
    for u in (0.1, 0.5, 0.93):
        a = oracle.sample_row(x, p, mask=wl.pack_mask(allow), mask_kind=MASK_ALLOW, u=u)
        b = oracle.sample_row(x, p, mask=wl.pack_mask(~allow), mask_kind=MASK_BAN, u=u)
        assert a["id"] == b["id"] and allow[a["id"]]


def test_ties_break_by_lowest_index(oracle):
    x = np.zeros(64, np.float32)
    x[[5, 9, 40]] = 1.0
    r = oracle.sample_row(x, params(greedy=True))
    assert r["id"] == 5
    r = oracle.sample_row(x, params(top_k=2), u=0.99, cap=2)
    assert list(r["tokens"]) == [5, 9] and r["id"] == 9
    x[3] = -0.0
    x[2] = 0.0
    r = oracle.sample_row(x, params(top_k=5), u=0.0, cap=5)
    assert list(r["tokens"]) == [5, 9, 40, 0, 1]  # -0 ties with +0: lowest index first


def test_nan_refused(oracle):
    x = np.ones(100, np.float32)
    x[17] = np.nan
    assert oracle.sample_row(x, params(greedy=True))["status"] == 4
    ban = np.zeros(100, bool)
    ban[17] = True
    assert oracle.sample_row(x, params(greedy=True), mask=wl.pack_mask(ban), mask_kind=MASK_BAN)["status"] == 0


# ---------------------------------------------------------------- randomized agreement with the reference
def test_random_agreement_with_reference(oracle, ref):
    rng = np.random.default_rng(2024)
    mismatch = []
    for trial in range(150):
        n = int(rng.choice([7, 64, 2048, 3072, 9000, 20000]))
        x = (rng.standard_normal(n) * rng.choice([1, 2, 3])).astype(np.float32)
        p = params(greedy=bool(rng.random() < 0.2), temperature=float(rng.choice([0.6, 0.9, 1.3])),
                   top_k=int(rng.choice([0, 1, 40, 50, 200, 5000])), top_p=float(rng.choice([1.0, 0.95, 0.5, 0.0])),
                   repetition_penalty=float(rng.choice([1.0, 1.05, 0.8, 1.3])))
        h = rng.integers(-2, n + 2, size=int(rng.integers(0, 600))).astype(np.int32)
        banned = rng.random(n) < 0.05
        u = float(rng.random())
        st1, id1 = ref.sample(x, p, h, banned, u)
        res = oracle.sample_row(x, p, h, wl.pack_mask(banned), MASK_BAN, u)
        if (st1, id1) != (res["status"], res["id"]):
            mismatch.append((trial, st1, id1, res["status"], res["id"]))
    assert not mismatch


def test_family_agreement_with_reference(oracle, ref):
    """haru::candidates and drama3::candidates of the restatement against the compiled reference on random
    rows (ties, -inf bans, top_k 0/1/beyond the vocabulary, top_p edges): identical statuses, tokens and
    weights."""
    rng = np.random.default_rng(77)
    for trial in range(120):
        n = int(rng.choice([1, 5, 300, 4096, 4097, 9000]))
        x = (rng.standard_normal(n) * rng.choice([0.5, 2, 8])).astype(np.float32)
        if rng.random() < 0.3:
            x = np.round(x).astype(np.float32)  # ties
        t = float(rng.choice([0.0, 1e-6, 0.5, 1.0, 1.7]))
        k = int(rng.choice([0, 1, 30, 500, n, n + 3]))
        p = float(rng.choice([0.0, 0.1, 0.9, 1.0]))
        xh = x.copy()
        if rng.random() < 0.3 and n > 2:
            xh[rng.choice(n, max(1, n // 10), replace=False)] = -np.inf
        for fam, xx in (("haru_candidates", xh), ("drama3_candidates", x)):
            a = getattr(oracle, fam)(xx, t, k, p)
            b = getattr(ref, fam)(xx, t, k, p)
            assert a[0] == b[0], (trial, fam)
            assert np.array_equal(a[1], b[1]), (trial, fam)
            assert np.array_equal(a[2], b[2]), (trial, fam)


# ---------------------------------------------------------------- Haru's DRY and logit shaping
@pytest.mark.parametrize("case", ["mild", "long-window", "allowed-1"])
def test_haru_dry_golden(oracle, case):
    """haru::Dry (haru/sampler.cpp:82-114) after every token of the fixture's stream, and shape_logits()
    (:116-124), as the compiled reference returned them: bit for bit."""
    from oracle import DryConfig
    c = load_cases("haru_dry_cases.npz")[case]
    cfg = DryConfig(*[float(v) for v in c["config"]], *[int(v) for v in c["ints"]], 0)
    ids = (0, 1, 2)
    pt, pv, cnt = oracle.dry_run(cfg, np.array(ids, np.int32), c["tokens"], c["pen_tokens"].shape[1])
    assert np.array_equal(cnt, c["counts"])
    assert np.array_equal(pt, c["pen_tokens"]) and np.array_equal(pv, c["pen_values"])
    for r in range(4):
        n = 100 * (r + 1)
        k = int(cnt[n - 1])
        got = oracle.haru_shape(c["logits"][r], pt[n - 1, :k], pv[n - 1, :k], c["silent"][r], *ids, 0.5 * r, r == 3)
        assert np.array_equal(got, c["shaped"][r], equal_nan=True)


def test_haru_dry_agreement_with_reference(oracle, ref):
    """Random streams with repeats, random settings: the restatement's penalties equal the reference's
    after every token."""
    from oracle import DryConfig
    rng = np.random.default_rng(404)
    for trial in range(40):
        cfg = DryConfig(float(rng.choice([0.5, 0.8, 1.0])), float(rng.choice([1.2, 1.75, 2.0])),
                        float(rng.choice([0.5, 3.0, 1e9])), int(rng.choice([0, 1, 2, 3, 5])),
                        int(rng.choice([0, 1, 8, 64, 300])), int(rng.choice([0, 1, 4, 16, 64])), 0)
        vocab = int(rng.choice([4, 20, 200]))
        toks = rng.integers(0, vocab, size=300).astype(np.int32)
        for _ in range(20):  # copied runs
            a, b = sorted(rng.integers(0, 300, size=2))
            L = int(rng.integers(2, 20))
            if b + L <= 300 and a + L <= b:
                toks[b:b + L] = toks[a:a + L]
        exempt = np.array(rng.choice(vocab, size=int(rng.integers(0, 3)), replace=False), np.int32)
        got = oracle.dry_run(cfg, exempt, toks, 128)
        want = ref.dry_run(cfg, exempt, toks, 128)
        for g, w in zip(got, want):
            assert np.array_equal(g, w), trial
