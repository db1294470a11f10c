"""Haru's DRY state and logit shaping on the device (ssb_dry_*, ssb_haru_shape_rows) against the compiled
reference's fixtures, the oracle's restatement of haru::Dry / shape_logits (haru/sampler.cpp:82-124), and
the reference itself over a whole decode loop.

Tolerances: penalty tokens and counts exact (integers); penalty values within 4 ulp relative (the
device's pow against glibc's, each within a couple of ulp; everything else is the same IEEE double
arithmetic); shaped logits and drawn ids exact."""
import os

import numpy as np
import pytest

import speech_sampler as ss
from oracle import DryConfig as ODryConfig, Oracle, RefSampler, ref_available

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
IDS = (0, 1, 2)  # pad, eop, eos
PEN_RTOL = 4 * 2.0 ** -52


def load_cases(name):
    z = np.load(os.path.join(GOLDEN, name))
    out = {}
    for key in z.files:
        case, field = key.split("/", 1) if "/" in key else ("", key)
        out.setdefault(case, {})[field] = z[key]
    return out


def torch_mod():
    import torch
    return torch


def _cfg(c):
    return ss.DryConfig(*[float(v) for v in c["config"]], *[int(v) for v in c["ints"]], 0)


def _ocfg(cfg):
    return ODryConfig(cfg.multiplier, cfg.base, cfg.max_penalty, cfg.allowed_length, cfg.lookback,
                      cfg.max_match_length, 0)


def _same_penalties(got, want_tok, want_val):
    t, v = got
    assert np.array_equal(t, want_tok), (t, want_tok)
    assert np.all(np.abs(v - want_val) <= PEN_RTOL * np.abs(want_val)), (v, want_val)


@pytest.mark.parametrize("case", ["mild", "long-window", "allowed-1"])
def test_dry_golden_on_device(engine, case):
    torch = torch_mod()
    c = load_cases("haru_dry_cases.npz")[case]
    dry = ss.Dry(engine, _cfg(c), 1, IDS)
    try:
        tok = torch.empty(1, dtype=torch.int32, device="cuda")
        for s, t in enumerate(c["tokens"]):
            tok.fill_(int(t))
            dry.update(tok)
            n = int(c["counts"][s])
            _same_penalties(dry.penalties(0), c["pen_tokens"][s, :n], c["pen_values"][s, :n])
    finally:
        dry.close()


def test_dry_many_streams_against_oracle(engine):
    """16 streams updated together, some skipping steps (token -1), each with its own copied runs; after
    every 25 steps every stream's penalties equal the oracle's over the tokens it took."""
    torch = torch_mod()
    orc = Oracle()
    rng = np.random.default_rng(9)
    streams, steps = 16, 300
    for cfg in (ss.DryConfig(0.8, 1.75, 3.0, 2, 64, 8, 0), ss.DryConfig(1.0, 2.0, 1e6, 3, 1000, 40, 0),
                ss.DryConfig(0.3, 1.1, 2.0, 1, 7, 3, 0)):
        toks = rng.integers(3, 40, size=(steps, streams)).astype(np.int32)
        for s in range(streams):
            for _ in range(15):
                a, b = sorted(rng.integers(0, steps, size=2))
                L = int(rng.integers(2, 25))
                if a + L <= b and b + L <= steps:
                    toks[b:b + L, s] = toks[a:a + L, s]
        toks[rng.random((steps, streams)) < 0.08] = 1          # an exempt id (EOP)
        toks[rng.random((steps, streams)) < 0.05] = -1         # the stream drew nothing this step
        dry = ss.Dry(engine, cfg, streams, IDS)
        try:
            dev = torch.from_numpy(toks).cuda()
            for step in range(steps):
                dry.update(dev[step])
                if step % 25 == 24 or step == steps - 1:
                    for s in range(streams):
                        taken = toks[:step + 1, s]
                        taken = taken[taken >= 0]
                        pt, pv, cnt = orc.dry_run(_ocfg(cfg), np.array(IDS, np.int32), taken, 2048)
                        n = int(cnt[-1]) if len(taken) else 0
                        _same_penalties(dry.penalties(s, cap=2048), pt[-1, :n] if n else pt[:0, 0],
                                        pv[-1, :n] if n else pv[:0, 0])
        finally:
            dry.close()


@pytest.mark.parametrize("case", ["mild", "long-window", "allowed-1"])
def test_shape_golden_on_device(engine, case):
    """shape_logits() of the fixture's rows: stream r has taken the first 100 (r + 1) tokens, row r's EOP
    bias is 0.5 r and row 3 must speak."""
    torch = torch_mod()
    c = load_cases("haru_dry_cases.npz")[case]
    dry = ss.Dry(engine, _cfg(c), 4, IDS)
    try:
        toks = np.full((400, 4), -1, np.int32)
        for r in range(4):
            toks[:100 * (r + 1), r] = c["tokens"][:100 * (r + 1)]
        dev = torch.from_numpy(toks).cuda()
        for step in range(400):
            dry.update(dev[step])
        silent = torch.from_numpy(c["silent"]).cuda()
        must = torch.tensor([0, 0, 0, 1], dtype=torch.int32, device="cuda")
        for r in range(4):
            x = torch.from_numpy(c["logits"]).cuda()
            ss.haru_shape(engine, x, silent, *IDS, eop_bias=0.5 * r, must_speak=must, dry=dry)
            got = x.cpu().numpy()[r]
            assert np.array_equal(got, c["shaped"][r]), np.nonzero(got != c["shaped"][r])
    finally:
        dry.close()


def test_haru_decode_loop_device_resident(engine):
    """The dialogue's text step (haru/dialogue.cpp:211-227) for 8 streams over 96 frames with nothing read
    back inside the loop: shape (DRY penalties, silent logits, EOP bias, must-speak on frame 0) ->
    Haru-family draw -> DRY update with the drawn ids, all queued on one stream. Against the reference
    itself run frame by frame on the host (shape_logits with its own Dry, haru::candidates, pick):
    identical ids at every frame. The logits favour a repeating pattern, so DRY changes draws."""
    if not ref_available():
        pytest.skip("oracle/_ref is not built")
    torch = torch_mod()
    ref = RefSampler()
    rng = np.random.default_rng(77)
    S, F, V = 8, 96, 4096
    cfg = ss.DryConfig(0.8, 1.75, 3.0, 2, 64, 8, 0)
    T, K, P = 0.9, 40, 0.95
    x = (rng.standard_normal((F, S, V)) * 1.5).astype(np.float32)
    for f in range(F):
        x[f, :, 3 + (f % 7)] += 5.0  # a period-7 phrase the model "wants" to repeat
    silent = (rng.standard_normal((F, S, 2)) - 1.0).astype(np.float32)
    must = np.zeros((F, S), np.int32)
    must[0] = 1
    u = rng.random((F, S))
    dx, ds, dm, du = (torch.from_numpy(a).cuda() for a in (x, silent, must, u))
    dry = ss.Dry(engine, cfg, S, IDS)
    ids = torch.empty((F, S), dtype=torch.int32, device="cuda")
    st = torch.empty((F, S), dtype=torch.int32, device="cuda")
    p = ss.params(temperature=T, top_k=K, top_p=P, flavor=ss.FLAVOR_HARU)
    try:
        for f in range(F):
            row = dx[f].clone()
            ss.haru_shape(engine, row, ds[f], *IDS, eop_bias=0.25, must_speak=dm[f], dry=dry)
            engine.sample(row, p, u=du[f], ids=ids[f], status=st[f])
            dry.update(ids[f])
        got = ids.cpu().numpy()
        assert np.all(st.cpu().numpy() == 0)
    finally:
        dry.close()
    exempt = np.array(IDS, np.int32)
    differ = 0
    for s in range(S):
        taken = []
        for f in range(F):
            shaped = ref.haru_shape(x[f, s], _ocfg(cfg), exempt, np.array(taken, np.int32), silent[f, s], *IDS, 0.25,
                                    bool(must[f, s]))
            hst, tok, w = ref.haru_candidates(shaped, T, K, P)
            assert hst == 0
            want = int(tok[ref.pick(w, u[f, s])])
            plain_st, plain_tok, plain_w = ref.haru_candidates(x[f, s], T, K, P)
            differ += want != int(plain_tok[ref.pick(plain_w, u[f, s])])
            assert got[f, s] == want, (f, s, got[f, s], want)
            taken.append(want)
    assert differ > 0  # shaping changed some draws: the test exercises it
