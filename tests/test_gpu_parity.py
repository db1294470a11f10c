"""Parity of the CUDA engine (through its C ABI) with the oracle restatement and the reference's golden
vectors. Token ids must be identical; a mismatch is tolerated only where the draw u lies within 1e-12
of a boundary between two candidates' cumulative shares (the reference's own device-vs-CPU policy,
checks/qwen3-tts/qwen3-tts-graph-sampler-check.cpp:40-44, with a far smaller margin) — none is
expected. Restricted (post-penalty) logits must be bit-identical (fp32 ops in the same order), and
candidate weights within 1e-12 relative (the north-star tolerance is 1e-5 for fp32, 1e-2 for bf16;
the only difference is CUDA's double exp against glibc's, each within 1 ulp)."""
import json
import os

import numpy as np
import pytest

import speech_sampler as ss
import speech_workloads as wl
from oracle import MASK_ALLOW, MASK_BAN, MASK_NONE, params

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
BOUNDARY = 1e-12
WEIGHT_RTOL = 1e-12


def torch_mod():
    import torch
    return torch


def dev(a, dtype=None):
    torch = torch_mod()
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.view(dtype)
    return t.cuda()


def engine_run(engine, logits, p, history=None, history_len=None, mask=None, mask_kind=MASK_NONE, u=None,
               row_params=None, max_top_k=0, cap=0, ld=None):
    """Runs the engine on host arrays; returns ids, status (and candidates when cap > 0)."""
    torch = torch_mod()
    if logits.dtype == np.uint16:
        x = dev(logits, torch.bfloat16)
    else:
        x = dev(logits.astype(np.float32))
    if ld is not None and ld != x.shape[1]:
        big = torch.zeros((x.shape[0], ld), dtype=x.dtype, device="cuda")
        big[:, :x.shape[1]] = x
        x = big[:, :x.shape[1]]
    h = None if history is None else dev(history.astype(np.int32))
    hl = None if history_len is None else dev(history_len.astype(np.int32))
    m = None if mask is None else dev(mask.view(np.int32))
    uu = None if u is None else dev(np.asarray(u, np.float64))
    rp = None if row_params is None else dev(ss.params_array(row_params).view(np.uint8)).view(torch.int32)
    if cap:
        ids, st, tok, w, cnt, proc = engine.candidates(x, p, h, hl, m, mask_kind, uu, rp, max_top_k, cap=cap)
        torch.cuda.synchronize()
        return (ids.cpu().numpy(), st.cpu().numpy(), tok.cpu().numpy(), w.cpu().numpy(), cnt.cpu().numpy(),
                proc.cpu().numpy())
    ids, st = engine.sample(x, p, h, hl, m, mask_kind, uu, rp, max_top_k)
    torch.cuda.synchronize()
    return ids.cpu().numpy(), st.cpu().numpy()


def boundary_distance(oracle, logits_row, p, history, mask, mask_kind, u):
    """Distance of u from the nearest cumulative-share boundary of the oracle's candidates."""
    r = oracle.sample_row(logits_row, p, history, mask, mask_kind, u, cap=logits_row.shape[-1])
    w = r["weights"]
    if len(w) < 2:
        return np.inf
    cum = np.cumsum(w / w.sum())[:-1]
    return float(np.min(np.abs(cum - u)))


def assert_ids(oracle, got_ids, got_st, want_ids, want_st, logits, p_of, hist_of, mask_of, mask_kind, u):
    assert np.array_equal(got_st, want_st), (np.nonzero(got_st != want_st)[0][:10], got_st[:10], want_st[:10])
    bad = np.nonzero(got_ids != want_ids)[0]
    near = 0
    for r in bad:
        d = boundary_distance(oracle, logits[r], p_of(r), hist_of(r), mask_of(r), mask_kind, u[r])
        assert d < BOUNDARY, f"row {r}: engine {got_ids[r]} oracle {want_ids[r]} u {u[r]} boundary distance {d}"
        near += 1
    return near


# ---------------------------------------------------------------- the reference's golden cases
def load_cases(name):
    z = np.load(os.path.join(GOLDEN, name))
    out = {}
    for key in z.files:
        case, field = key.split("/", 1) if "/" in key else ("", key)
        out.setdefault(case, {})[field] = z[key]
    return out


@pytest.mark.parametrize("case", sorted(load_cases("qwen3_tts_cases.npz")))
def test_golden_qwen3_tts(engine, case):
    c = load_cases("qwen3_tts_cases.npz")[case]
    settings = json.loads(str(c["settings"]))
    stack = settings.pop("stack")
    p = ss.params(**settings)
    rows, n_u = c["u"].shape
    vocab = c["logits"].shape[1]
    # one engine row per (row, u)
    x = np.repeat(c["logits"], n_u, axis=0)
    hist = np.repeat(c["history"], n_u, axis=0)
    mask = np.repeat(wl.pack_mask(c["banned"]), n_u, axis=0) if stack == "talker" else None
    ids, st, tok, w, cnt, _ = engine_run(engine, x, p, hist, None, mask, MASK_BAN if mask is not None else MASK_NONE,
                                         c["u"].reshape(-1), cap=64)
    assert np.array_equal(st.reshape(rows, n_u), c["status"])
    assert np.array_equal(ids.reshape(rows, n_u), c["ids"]), case
    if not p.greedy:
        for r in range(rows):
            e = r * n_u
            n = int(c["cand_count"][r])
            assert cnt[e] == n
            m = min(n, 64)
            wr = c["cand_weights"][r, :m]
            pos = wr > 0
            assert np.array_equal(tok[e, :m][pos], c["cand_tokens"][r, :m][pos])
            np.testing.assert_allclose(w[e, :m], wr, rtol=WEIGHT_RTOL, atol=0)


def test_golden_kats(engine):
    k = json.load(open(os.path.join(GOLDEN, "kat.json")))
    x = np.array([[1.0, 2.0], [1.0, 2.0]], np.float32)
    h = np.array([[0, 1], [0, 1]], np.int32)
    for greedy in (True, False):
        ids, st = engine_run(engine, x, ss.params(greedy=greedy, repetition_penalty=1e-40), h, u=[0.5, 0.5])
        assert list(st) == [k["penalty_1e-40_status"][0]] * 2 == [ss.ROW_PENALTY_OVERFLOW] * 2
        assert list(ids) == [-1, -1]
    row = np.random.default_rng(k["temperature_1e-38_row_seed"]).standard_normal(2048, dtype=np.float32) * np.float32(1.5)
    ids, st = engine_run(engine, row[None], ss.params(temperature=1e-38, top_k=50), u=[0.5])
    assert st[0] == k["temperature_1e-38_status"] == ss.ROW_TEMPERATURE_OVERFLOW
    # pick() at the edges of the cumulative shares: logits ln(4), ln(3), ln(2), ln(1) at temperature 1
    # are candidates in index order with shares 0.4, 0.3, 0.2, 0.1; the engine agrees with the oracle
    # at every edge of the reference's check, including draws exactly on a share.
    lw = np.log(np.array([4, 3, 2, 1], np.float64)).astype(np.float32)
    edges = k["pick_edges"] + [0.4, 0.7, 0.9, 0.39999, 0.70001]
    from oracle import Oracle
    o = Oracle()
    for e in edges:
        ids, st = engine_run(engine, lw[None], ss.params(), u=[e])
        assert st[0] == 0 and ids[0] == o.sample_row(lw, params(), u=e)["id"], e


# ---------------------------------------------------------------- small vocabularies vs the oracle
def random_cases(seed, n_cases, vocabs):
    rng = np.random.default_rng(seed)
    for i in range(n_cases):
        v = int(rng.choice(vocabs))
        b = int(rng.choice([1, 3, 17, 64]))
        bf16 = bool(rng.random() < 0.3)
        x = (rng.standard_normal((b, v)) * rng.choice([1.0, 2.0, 3.0])).astype(np.float32)
        if bf16:
            x = wl.to_bf16_bits(x)
        kw = dict(greedy=bool(rng.random() < 0.15), temperature=float(rng.choice([0.5, 0.9, 1.0, 1.7])),
                  top_k=int(rng.choice([0, 1, 2, 40, 50, 300, v + 5])), top_p=float(rng.choice([1.0, 0.95, 0.5, 0.0])),
                  repetition_penalty=float(rng.choice([1.0, 1.05, 0.8])),
                  presence_penalty=float(rng.choice([0.0, 0.0, 0.5])), frequency_penalty=float(rng.choice([0.0, 0.3])))
        hl = int(rng.choice([0, 5, 64, 700]))
        hist = rng.integers(-3, v + 3, size=(b, max(hl, 1))).astype(np.int32) if hl else None
        kind = int(rng.choice([MASK_NONE, MASK_BAN, MASK_ALLOW]))
        dens = float(rng.choice([0.01, 0.2, 0.7]))
        mask = wl.pack_mask(rng.random((b, v)) < dens) if kind != MASK_NONE else None
        u = rng.random(b, dtype=np.float32).astype(np.float64)
        yield i, x, kw, hist, mask, kind, u


@pytest.mark.parametrize("vocabs", [[7, 100, 2048, 3072], [5000, 8192]])
def test_small_vocab_random_vs_oracle(engine, oracle, vocabs):
    near = 0
    for i, x, kw, hist, mask, kind, u in random_cases(len(vocabs) * 7 + vocabs[0], 40, vocabs):
        p = ss.params(**kw)
        op = params(**kw)
        want_ids, want_st, want_proc = oracle.sample_rows(x, op, history=hist, mask=mask, mask_kind=kind, u=u,
                                                          want_processed=True)
        ids, st, tok, w, cnt, proc = engine_run(engine, x, p, hist, None, mask, kind, u, cap=16)
        near += assert_ids(oracle, ids, st, want_ids, want_st, x, lambda r: op,
                           lambda r: None if hist is None else hist[r], lambda r: None if mask is None else mask[r], kind, u)
        ok = want_st == 0
        assert np.array_equal(proc[ok].view(np.uint32), want_proc[ok].view(np.uint32)), f"case {i}: restricted logits differ"
        for r in np.nonzero(ok)[0][:4]:
            o = oracle.sample_row(x[r], op, None if hist is None else hist[r], None if mask is None else mask[r], kind,
                                  u[r], cap=16)
            assert cnt[r] == o["count"]
            m = min(16, o["count"])
            assert np.array_equal(tok[r, :m], o["tokens"][:m])
            np.testing.assert_allclose(w[r, :m], o["weights"][:m], rtol=WEIGHT_RTOL)
    assert near == 0


# ---------------------------------------------------------------- large vocabularies (streaming kernel)
def test_config1_greedy_suppress(engine, oracle):
    c = wl.config1(rows=64)
    want, wst, _ = oracle.sample_rows(c["logits"], params(greedy=True), mask=c["mask"], mask_kind=MASK_BAN)
    for b in (1, 64):
        ids, st = engine_run(engine, c["logits"][:b], ss.params(greedy=True), mask=c["mask"], mask_kind=MASK_BAN)
        assert np.array_equal(ids, want[:b]) and np.all(st == 0)
    g = load_cases("large_vocab_cases.npz")["config1"]
    cg = wl.config1(rows=int(g["rows"]))  # the golden rows (the generator's draws depend on the row count)
    ids, st = engine_run(engine, cg["logits"], ss.params(greedy=True), mask=cg["mask"], mask_kind=MASK_BAN)
    assert np.array_equal(ids, g["ids"])


@pytest.mark.parametrize("rows", [1, 8, 32, 256])
def test_config4_text_decoder(engine, oracle, rows):
    c = wl.config4(rows=rows)
    kw = c["params"]
    want, wst, _ = oracle.sample_rows(c["logits_bf16"], params(**kw), history=c["history"], u=c["u"])
    ids, st = engine_run(engine, c["logits_bf16"], ss.params(**kw), c["history"], u=c["u"])
    near = assert_ids(oracle, ids, st, want, wst, c["logits_bf16"], lambda r: params(**kw), lambda r: c["history"][r],
                      lambda r: None, MASK_NONE, c["u"])
    assert near == 0


def test_config4_candidates_and_processed(engine, oracle):
    c = wl.config4(rows=4)
    kw = c["params"]
    ids, st, tok, w, cnt, proc = engine_run(engine, c["logits_bf16"], ss.params(**kw), c["history"], u=c["u"], cap=40)
    for r in range(4):
        o = oracle.sample_row(c["logits_bf16"][r], params(**kw), c["history"][r], u=c["u"][r], cap=40, want_processed=True)
        assert np.array_equal(proc[r].view(np.uint32), o["processed"].view(np.uint32))
        assert cnt[r] == o["count"]
        assert np.array_equal(tok[r, :o["count"]], o["tokens"])
        np.testing.assert_allclose(w[r, :o["count"]], o["weights"], rtol=WEIGHT_RTOL)


@pytest.mark.parametrize("rows,vocab,kw", [
    (1, 151936, dict(temperature=0.8, top_k=40, top_p=0.95)),
    (3, 151937, dict(temperature=1.3, top_k=200, top_p=0.9, repetition_penalty=1.2)),   # ragged tail
    (5, 50000, dict(temperature=0.6, top_k=1024, top_p=1.0)),                          # the largest streamed k
    (2, 9000, dict(temperature=0.9, top_k=3, top_p=0.0, presence_penalty=1.0)),         # top-p 0 keeps one
    (4, 20011, dict(greedy=True, repetition_penalty=1.3)),
])
def test_stream_variants(engine, oracle, rows, vocab, kw):
    rng = np.random.default_rng(rows * 1000 + vocab)
    x = (rng.standard_normal((rows, vocab)) * 2).astype(np.float32)
    hist = rng.integers(-2, vocab + 2, size=(rows, 300)).astype(np.int32)
    hist[:, :50] = hist[:, 50:100]  # duplicates
    hlen = rng.integers(0, 301, size=rows).astype(np.int32)
    ban = rng.random((rows, vocab)) < 0.05
    u = rng.random(rows, dtype=np.float32).astype(np.float64)
    op = params(**kw)
    want_ids, want_st = [], []
    for r in range(rows):
        o = oracle.sample_row(x[r], op, hist[r, :hlen[r]], wl.pack_mask(ban[r]), MASK_BAN, u[r])
        want_ids.append(o["id"])
        want_st.append(o["status"])
    for ld in (vocab, vocab + 1):  # vectorized and scalar (unaligned) loads
        ids, st = engine_run(engine, x, ss.params(**kw), hist, hlen, wl.pack_mask(ban), MASK_BAN, u, ld=ld)
        assert np.array_equal(st, want_st)
        assert np.array_equal(ids, want_ids), (ld, ids, want_ids)


def _one_warp_allow(rows, vocab, g):
    """Allow mask keeping only the columns whose 16-byte group i has i % 256 < 32: in a one-CTA row of the
    top-k kernel those are the groups of the first consumer warp (group i goes to consumer lane i % 256),
    so every other warp sees only masked tokens."""
    cols = np.arange(vocab)
    return np.broadcast_to(((cols // g) % 256) < 32, (rows, vocab))


@pytest.mark.parametrize("bf16", [False, True])
@pytest.mark.parametrize("shape", ["one-warp-allow", "ascending", "negative-temperature"])
def test_topk_rare_paths(engine, oracle, bf16, shape):
    """Rows that no random batch produces, 160 of them (one CTA per row): allowed tokens that only one
    consumer warp streams, a row whose logits rise from its first column to its last (every block a new
    maximum), and a negative temperature (the order reversed, so no raw bound applies)."""
    rows, vocab = 160, 151936
    rng = np.random.default_rng(7 + bf16 + 10 * len(shape))
    x = (rng.standard_normal((rows, vocab)) * 3).astype(np.float32)
    mask, kind = None, MASK_NONE
    kw = dict(temperature=0.8, top_k=40, top_p=0.95, presence_penalty=0.5, frequency_penalty=0.3)
    if shape == "one-warp-allow":
        mask, kind = wl.pack_mask(_one_warp_allow(rows, vocab, 8 if bf16 else 4)), MASK_ALLOW
    elif shape == "ascending":
        x = (np.linspace(-20, 20, vocab, dtype=np.float32)[None, :] + 1e-3 * x).astype(np.float32)
    else:
        kw = dict(temperature=-0.7, top_k=40, top_p=0.9, repetition_penalty=1.1)
    logits = wl.to_bf16_bits(x) if bf16 else x
    hist = rng.integers(0, vocab, size=(rows, 256)).astype(np.int32)
    u = rng.random(rows)
    want, wst, _ = oracle.sample_rows(logits, params(**kw), history=hist, mask=mask, mask_kind=kind, u=u)
    ids, st = engine_run(engine, logits, ss.params(**kw), hist, mask=mask, mask_kind=kind, u=u)
    near = assert_ids(oracle, ids, st, want, wst, logits, lambda r: params(**kw), lambda r: hist[r],
                      lambda r: None if mask is None else mask[r], kind, u)
    assert near == 0


def test_row_params_mixed(engine, oracle):
    rng = np.random.default_rng(7)
    rows, vocab = 6, 151936
    x = (rng.standard_normal((rows, vocab)) * 2).astype(np.float32)
    plist = [dict(greedy=True), dict(temperature=0.7, top_k=50), dict(temperature=1.1, top_k=10, top_p=0.8),
             dict(greedy=True, repetition_penalty=1.5), dict(temperature=0.9, top_k=64, frequency_penalty=0.2),
             dict(temperature=0.9, top_k=100)]
    hist = rng.integers(0, vocab, size=(rows, 64)).astype(np.int32)
    u = rng.random(rows, dtype=np.float32).astype(np.float64)
    want = [oracle.sample_row(x[r], params(**plist[r]), hist[r], u=u[r])["id"] for r in range(rows)]
    ids, st = engine_run(engine, x, ss.params(), hist, u=u, row_params=[ss.params(**q) for q in plist], max_top_k=100)
    assert np.array_equal(ids, want) and np.all(st == 0)
    ids, st = engine_run(engine, x, ss.params(), hist, u=u, row_params=[ss.params(**q) for q in plist], max_top_k=50)
    assert st[5] == ss.ROW_INVALID_ROW and st[2] == 0 and ids[5] == -1


@pytest.mark.parametrize("vocab", [3072, 151936])
def test_statuses(engine, vocab):
    rng = np.random.default_rng(vocab)
    x = rng.standard_normal((6, vocab)).astype(np.float32)
    x[0, 17] = np.nan                     # NaN, unmasked -> NON_FINITE_INPUT
    x[1, 18] = np.nan                     # NaN under the ban -> fine
    x[3, 5] = np.inf                      # +inf with a penalty -> PENALTY_OVERFLOW
    ban = np.zeros((6, vocab), bool)
    ban[1, 18] = True
    ban[2, :] = True                      # every token banned -> NO_FINITE_LOGIT
    h = np.zeros((6, 4), np.int32)
    p = ss.params(temperature=0.9, top_k=20, repetition_penalty=1.1)
    ids, st = engine_run(engine, x, p, h, mask=wl.pack_mask(ban), mask_kind=MASK_BAN, u=np.full(6, 0.3))
    assert list(st) == [ss.ROW_NON_FINITE_INPUT, 0, ss.ROW_NO_FINITE_LOGIT, ss.ROW_PENALTY_OVERFLOW, 0, 0]
    assert ids[0] == -1 and ids[2] == -1 and ids[1] >= 0
    from oracle import Oracle
    o = Oracle()
    for t in (0.0, 1e-38, -1.0, float("inf")):  # degenerate temperatures: statuses as the oracle defines them
        ids, st = engine_run(engine, x[4:6], ss.params(temperature=t, top_k=20), u=np.full(2, 0.3))
        want = [o.sample_row(x[r], params(temperature=t, top_k=20), u=0.3) for r in (4, 5)]
        assert list(st) == [w["status"] for w in want], t
        assert list(ids) == [w["id"] for w in want], t
    ids, st = engine_run(engine, x[4:6], ss.params(temperature=0.0, top_k=20), u=np.full(2, 0.3))
    assert list(st) == [ss.ROW_TEMPERATURE_OVERFLOW] * 2


@pytest.mark.parametrize("vocab", [100, 3072, 151936])  # 3072: more than 512 ties at the small kernel's bound
def test_ties_lowest_index(engine, oracle, vocab):
    x = np.zeros((3, vocab), np.float32)
    x[0, [11, 7, 99 % vocab]] = 1.0
    x[2, :] = -0.0
    x[2, ::2] = 0.0
    u = np.array([0.999, 0.999, 0.5])
    for kw in (dict(greedy=True), dict(top_k=2), dict(top_k=50, temperature=3.0)):
        want = [oracle.sample_row(x[r], params(**kw), u=u[r])["id"] for r in range(3)]
        ids, st = engine_run(engine, x, ss.params(**kw), u=u)
        assert np.array_equal(ids, want), kw
    xb = wl.to_bf16_bits(np.round(np.random.default_rng(1).standard_normal((4, vocab)) * 2) / 2)  # many ties
    u4 = np.array([0.1, 0.4, 0.7, 0.95])
    want = [oracle.sample_row(xb[r], params(top_k=40, temperature=0.8), u=u4[r])["id"] for r in range(4)]
    ids, st = engine_run(engine, xb, ss.params(top_k=40, temperature=0.8), u=u4)
    assert np.array_equal(ids, want)


def test_repeat_launches_and_host_entry(engine, oracle):
    """Split-row counters reset themselves: repeated launches agree; the host-buffer entry point agrees."""
    torch = torch_mod()
    c = wl.config4(rows=2)
    kw = c["params"]
    first = None
    for _ in range(5):
        ids, st = engine_run(engine, c["logits_bf16"], ss.params(**kw), c["history"], u=c["u"])
        first = ids if first is None else first
        assert np.array_equal(ids, first)
    ids_h, st_h = engine.sample_host(c["logits_bf16"], ss.params(**kw), c["history"], None, None, MASK_NONE, c["u"])
    assert np.array_equal(ids_h, first) and np.all(st_h == 0)
    torch.cuda.synchronize()


def test_draw_at_exact_boundaries(engine, oracle):
    """u placed exactly on pick()'s running sums (added as the reference adds them, in order): the
    parallel draw cannot decide such rows within its margin and defers to the sequential replay."""
    c = wl.config4(rows=8)
    kw = c["params"]
    p = params(**kw)
    us = []
    for r in range(8):
        o = oracle.sample_row(c["logits_bf16"][r], p, c["history"][r], None, MASK_NONE, 0.5, cap=128)
        w = [float(x) for x in o["weights"][:o["count"]]]
        total = 0.0
        for x in w:
            total += x
        cum, cums = 0.0, []
        for x in w[:-1]:
            cum += x / total
            cums.append(cum)
        us.append(cums[r % len(cums)] if cums else 0.5)
    u = np.array(us)
    ids, st = engine_run(engine, c["logits_bf16"], ss.params(**kw), c["history"], u=u)
    want, wst, _ = oracle.sample_rows(c["logits_bf16"], p, history=c["history"], u=u)
    assert_ids(oracle, ids, st, want, wst, c["logits_bf16"], lambda r: p, lambda r: c["history"][r], lambda r: None,
               MASK_NONE, u)


def test_context_mask_is_generation_banned(engine):
    """The talker's suppress mask of Generation::banned (qwen3-tts/sampler.cpp:62-67: the last 1024 ids but
    the end of speech 2150, and 2150 itself before frame 2) copied once into the context
    (ssb_context_mask) and used from there by ssb_sample_rows: the same ids as the same mask passed as a
    tensor, and no banned id drawn."""
    import ctypes
    import torch
    lib = engine.lib
    V, eos, suppressed, min_frames = wl.TALKER_VOCAB, 2150, 1024, 2

    def banned(frames):
        b = np.zeros(V, bool)
        b[V - suppressed:] = True
        b[eos] = frames < min_frames
        return b

    t = wl.config2(steps=16)
    p = ss.params(**t["params"])
    x = dev(t["logits"])
    x[:, eos] += 6.0  # the end of speech would win where allowed
    h, u = dev(t["history"]), dev(t["u"])
    for frames in (0, 5):
        words = np.ascontiguousarray(wl.pack_mask(banned(frames)), np.uint32)
        out = ctypes.c_void_p()
        assert lib.ssb_context_mask(engine.ctx, ctypes.c_void_p(words.ctypes.data), len(words), ctypes.byref(out)) == ss.OK
        ids_t, st_t = engine.sample(x, p, h, None, dev(words.view(np.int32)), MASK_BAN, u)
        ids = torch.empty(16, dtype=torch.int32, device="cuda")
        st = torch.empty(16, dtype=torch.int32, device="cuda")
        r = ss.Sampler._rows_struct(x, p, h, None, None, MASK_NONE, u, ids, st)
        r.mask, r.mask_ld, r.mask_kind = out.value, 0, MASK_BAN
        assert lib.ssb_sample_rows(engine.ctx, ctypes.byref(r), None) == ss.OK
        torch.cuda.synchronize()
        assert torch.equal(ids, ids_t) and torch.equal(st, st_t) and bool(torch.all(st == 0))
        got = ids.cpu().numpy()
        assert not banned(frames)[got].any()
        assert (got == eos).any() == (frames >= min_frames)
    assert lib.ssb_context_mask(engine.ctx, ctypes.c_void_p(words.ctypes.data), 0, ctypes.byref(out)) == ss.OUT_OF_RANGE
