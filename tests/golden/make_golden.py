"""Generates the golden fixtures under tests/golden/ from the REFERENCE'S OWN SAMPLER, compiled from its
sources into oracle/_ref/libref_sampler.so (oracle/Makefile). The reference ships no vectors for this
path (its generators, reference/qwen3-tts/sampling_cases.py and reference/haru/sampling_cases.py, need
model dumps), so the inputs here are seeded synthetic logits shaped like those cases, and the outputs
are what the reference's sample(), candidates(), pick(), uniform(), haru::candidates(),
drama3::candidates(), haru::Dry and shape_logits() return.

Run here, where the reference sources exist:   python tests/golden/make_golden.py
The fixtures travel with the repository; the tests never need the reference at run time.

Extension features the reference lacks (presence/frequency penalties, allow-masks, bf16, lowest-index
ties) are not in these fixtures: they are covered by the oracle restatement's own tests.
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "speech.cpp_b200"))

from oracle import RefSampler, build, params  # noqa: E402
import speech_workloads as wl  # noqa: E402

# Qwen3-TTS's talker: 3072 codes, end of speech 2150, the last 1024 ids suppressed except it, the end of
# speech banned for the first 2 frames (Generation::banned, src/families/qwen3-tts/sampler.cpp:62-67).
TALKER_VOCAB, CP_VOCAB, EOS, SUPPRESSED, MIN_FRAMES = 3072, 2048, 2150, 1024, 2
TALKER_FILE = dict(greedy=False, temperature=0.9, top_k=50, top_p=1.0, repetition_penalty=1.05)
CP_FILE = dict(greedy=False, temperature=0.9, top_k=50, top_p=1.0, repetition_penalty=1.0)

# The settings of the reference's sampling cases (reference/qwen3-tts/sampling_cases.py:79-94).
CASES = {
    "talker-file": ("talker", TALKER_FILE),
    "talker-top-p": ("talker", dict(temperature=1.3, top_k=0, top_p=0.8, repetition_penalty=1.2)),
    "talker-top-p-wide": ("talker", dict(temperature=2.5, top_k=0, top_p=0.99, repetition_penalty=1.05)),
    "talker-top-k-1": ("talker", dict(temperature=0.7, top_k=1, top_p=1.0, repetition_penalty=1.05)),
    "talker-top-p-0": ("talker", dict(temperature=0.9, top_k=0, top_p=0.0, repetition_penalty=1.05)),
    "talker-penalty-below-1": ("talker", dict(temperature=1.0, top_k=100, top_p=0.95, repetition_penalty=0.8)),
    "talker-greedy": ("talker", dict(greedy=True, temperature=0.9, top_k=50, top_p=1.0, repetition_penalty=1.5)),
    "code-predictor-file": ("code_predictor", CP_FILE),
    "code-predictor-top-p": ("code_predictor", dict(temperature=0.6, top_k=0, top_p=0.5, repetition_penalty=1.0)),
    "code-predictor-top-p-wide": ("code_predictor", dict(temperature=2.0, top_k=200, top_p=0.95, repetition_penalty=1.0)),
    "code-predictor-top-k-beyond-vocab": ("code_predictor", dict(temperature=1.1, top_k=5000, top_p=1.0, repetition_penalty=1.0)),
    "code-predictor-penalty": ("code_predictor", dict(temperature=0.9, top_k=50, top_p=1.0, repetition_penalty=1.3)),
    "code-predictor-greedy": ("code_predictor", dict(greedy=True, temperature=0.9, top_k=50, top_p=1.0, repetition_penalty=1.0)),
}
ROWS, N_U, CAP = 6, 8, 64


def talker_banned(frames: int) -> np.ndarray:
    b = np.zeros(TALKER_VOCAB, bool)
    b[TALKER_VOCAB - SUPPRESSED:] = True
    b[EOS] = frames < MIN_FRAMES
    return b


def qwen3_tts_cases(ref: RefSampler) -> dict:
    out = {}
    for ci, (name, (stack, settings)) in enumerate(CASES.items()):
        rng = np.random.default_rng(100 + ci)
        talker = stack == "talker"
        vocab = TALKER_VOCAB if talker else CP_VOCAB
        p = params(**settings)
        logits = (rng.standard_normal((ROWS, vocab), dtype=np.float32) * np.float32(2.0 if talker else 1.5))
        # histories: the talker's first codes of the frames before; the code predictor's codes of its frame
        hist = np.full((ROWS, 16), -1, np.int32)
        for r in range(ROWS):
            n = r * 3 if talker else min(r * 2, 15)
            hist[r, :n] = rng.integers(0, vocab, size=n)
            if r % 2 == 1 and n > 2:
                hist[r, 1] = hist[r, 0]  # a repeated id: the penalty applies once
        banned = np.stack([talker_banned(int((hist[r] >= 0).sum())) if talker else np.zeros(vocab, bool)
                           for r in range(ROWS)])
        u = np.empty((ROWS, N_U))
        u[:, :N_U // 2] = (np.arange(N_U // 2) + 0.5) / (N_U // 2)
        u[:, N_U // 2:] = rng.random((ROWS, N_U // 2), dtype=np.float32)
        ids = np.empty((ROWS, N_U), np.int32)
        status = np.empty((ROWS, N_U), np.int32)
        cand_tok = np.full((ROWS, CAP), -1, np.int32)
        cand_w = np.zeros((ROWS, CAP))
        cand_n = np.zeros(ROWS, np.int32)
        for r in range(ROWS):
            h = hist[r][hist[r] >= 0]
            for j in range(N_U):
                status[r, j], ids[r, j] = ref.sample(logits[r], p, h, banned[r] if talker else None, u[r, j])
            if not p.greedy:
                st, t, w = ref.candidates(logits[r], p, h, banned[r] if talker else None)
                cand_n[r] = len(t)
                cand_tok[r, :min(CAP, len(t))] = t[:CAP]
                cand_w[r, :min(CAP, len(t))] = w[:CAP]
        out[name] = dict(logits=logits, history=hist, banned=banned, u=u, ids=ids, status=status,
                         cand_tokens=cand_tok, cand_weights=cand_w, cand_count=cand_n,
                         settings=np.array(json.dumps(dict(stack=stack, **settings))))
    return out


def large_vocab_cases(ref: RefSampler) -> dict:
    """Shapes of the large-vocabulary configs, at few rows, regenerated from their seeds by the tests."""
    out = {}
    c1 = wl.config1(rows=4)
    ids = np.array([ref.sample(c1["logits"][r], params(greedy=True), None, c1["banned"])[1] for r in range(4)], np.int32)
    out["config1"] = dict(rows=np.int32(4), ids=ids)
    c4 = wl.config4(rows=3)
    x4 = wl.bf16_bits_to_f32(c4["logits_bf16"])
    p4 = params(temperature=0.8, top_k=40, top_p=0.95, repetition_penalty=1.1)  # reference features only
    res = [ref.sample(x4[r], p4, c4["history"][r], None, c4["u"][r]) for r in range(3)]
    out["config4_rep"] = dict(rows=np.int32(3), ids=np.array([x[1] for x in res], np.int32),
                              status=np.array([x[0] for x in res], np.int32))
    c5 = wl.config5(rows=3, density=0.01)
    p5 = params(temperature=1.0, top_k=0, top_p=0.9)
    res = [ref.sample(c5["logits"][r], p5, None, ~c5["allow"][r], c5["u"][r]) for r in range(3)]
    out["config5_d0.01"] = dict(rows=np.int32(3), density=np.float64(0.01),
                                ids=np.array([x[1] for x in res], np.int32),
                                status=np.array([x[0] for x in res], np.int32))
    return out


def kats(ref: RefSampler) -> dict:
    """Known answers of the reference's own checks (checks/qwen3-tts/qwen3-tts-sampler-check.cpp:70-116,
    checks/qwen3-tts/qwen3-tts-graph-sampler-check.cpp:163-186), recomputed by the reference itself."""
    weights = [1.0, 2.0, 3.0, 4.0]
    edges = [0.0, 0.0999, 0.1, 0.2999, 0.3000001, 0.65, 1.0]
    k = dict(pick_weights=weights, pick_edges=edges, pick_results=[ref.pick(weights, e) for e in edges],
             pick_single=ref.pick([5.0], 1.0))
    draws = ref.uniform(1, 400000)
    k["uniform_seed1_first16"] = [float(x).hex() for x in draws[:16]]
    counts = np.bincount([ref.pick(weights, x) for x in draws], minlength=4)
    k["uniform_seed1_shares"] = (counts / len(draws)).tolist()
    st = []
    for greedy in (True, False):
        p = params(greedy=greedy, repetition_penalty=1e-40)
        st.append(ref.sample(np.array([1.0, 2.0], np.float32), p, np.array([0, 1], np.int32), None, 0.5)[0])
    k["penalty_1e-40_status"] = st
    row = np.random.default_rng(9).standard_normal(2048, dtype=np.float32) * np.float32(1.5)
    k["temperature_1e-38_status"] = ref.sample(row, params(temperature=1e-38, top_k=50), None, None, 0.5)[0]
    k["temperature_1e-38_row_seed"] = 9
    return k


def haru_cases(ref: RefSampler) -> dict:
    out = {}
    rng = np.random.default_rng(11)
    x = rng.standard_normal((4, 4096), dtype=np.float32) * np.float32(2.0)
    x[1, rng.choice(4096, 100, replace=False)] = -np.inf  # banned tokens of the session
    for name, (t, k, p) in {"default": (0.7, 25, 1.0), "top-p": (0.7, 0, 0.9), "greedy": (0.0, 25, 1.0),
                            "wide": (1.5, 500, 0.95)}.items():
        toks = np.full((4, 600), -1, np.int32)
        ws = np.zeros((4, 600))
        ns = np.zeros(4, np.int32)
        for r in range(4):
            st, tk, w = ref.haru_candidates(x[r], t, k, p, cap=600)
            ns[r] = len(tk)
            toks[r, :len(tk)] = tk
            ws[r, :len(tk)] = w
        out[name] = dict(t=np.float32(t), k=np.int32(k), p=np.float32(p), tokens=toks, weights=ws, count=ns)
    out["logits"] = x
    return out


# The settings of the reference's Drama 3 sampling cases (reference/drama3/sampling_cases.py:32-43): the
# model card's, and cases around it; main-token rows span the end id and 4096 semantic ids (4097), the
# residual codebooks' heads 4096 codes.
DRAMA3_CASES = {
    "card": (4097, 1.0, 30, 0.9),
    "main-top-k-1": (4097, 1.0, 1, 0.9),
    "codes-top-p-narrow": (4096, 1.0, 30, 0.1),
    "codes-cold": (4096, 0.5, 30, 0.9),
    "codes-hot": (4096, 1.5, 100, 1.0),
    "main-every-token": (4097, 1.0, 4097, 1.0),
}
DRAMA3_ROWS = 4


def drama3_cases(ref: RefSampler) -> dict:
    """drama3::candidates() on seeded logits of each case's shape, and pick() of its weights with
    seeded draws: tokens, weights (exp(s - top), not normalized), counts and the ids."""
    out = {}
    rng = np.random.default_rng(23)
    for name, (n, t, k, p) in DRAMA3_CASES.items():
        x = (rng.standard_normal((DRAMA3_ROWS, n), dtype=np.float32) * np.float32(rng.choice([1.5, 3.0, 6.0])))
        u = rng.random(DRAMA3_ROWS)
        cap = min(k, n)
        toks = np.full((DRAMA3_ROWS, cap), -1, np.int32)
        ws = np.zeros((DRAMA3_ROWS, cap))
        ns = np.zeros(DRAMA3_ROWS, np.int32)
        ids = np.zeros(DRAMA3_ROWS, np.int32)
        for r in range(DRAMA3_ROWS):
            st, tk, w = ref.drama3_candidates(x[r], t, k, p, cap=cap)
            assert st == 0
            ns[r] = len(tk)
            toks[r, :len(tk)] = tk
            ws[r, :len(tk)] = w
            ids[r] = tk[ref.pick(w, u[r])]
        out[name] = dict(logits=x, t=np.float32(t), k=np.int32(k), p=np.float32(p), u=u, tokens=toks, weights=ws,
                         count=ns, ids=ids)
    return out


# DRY settings for the Haru fixtures (the file's dry_* keys, haru/sampler.cpp:63-73; the model's own values
# come with its GGUF, so these are seeded stand-ins of the same kind) and the text ids they exempt.
HARU_DRY = {"mild": (0.8, 1.75, 3.0, 2, 64, 8), "long-window": (1.0, 2.0, 50.0, 3, 512, 32),
            "allowed-1": (0.5, 1.5, 1.0, 1, 16, 4)}
HARU_IDS = (0, 1, 2)  # pad, eop, eos
HARU_DRY_STEPS, HARU_DRY_CAP = 400, 64


def haru_dry_tokens(rng, steps, vocab):
    """A token stream with the repeats DRY looks for: runs copied from earlier, interleaved with fresh
    tokens and the exempt text ids."""
    out = []
    while len(out) < steps:
        r = rng.random()
        if r < 0.45 and len(out) > 8:
            start = int(rng.integers(0, len(out) - 4))
            out.extend(out[start:start + int(rng.integers(2, 12))])
        elif r < 0.55:
            out.append(int(rng.choice(HARU_IDS)))
        else:
            out.extend(int(t) for t in rng.integers(3, vocab, size=int(rng.integers(1, 6))))
    return np.array(out[:steps], np.int32)


def haru_dry_cases(ref: RefSampler) -> dict:
    """haru::Dry's penalties after every token of seeded streams, and shape_logits() of seeded rows."""
    from oracle import DryConfig
    out = {}
    rng = np.random.default_rng(31)
    for name, c in HARU_DRY.items():
        cfg = DryConfig(*c, 0)
        toks = haru_dry_tokens(rng, HARU_DRY_STEPS, 60)
        pt, pv, cnt = ref.dry_run(cfg, np.array(HARU_IDS, np.int32), toks, HARU_DRY_CAP)
        x = (rng.standard_normal((4, 4096)) * 2).astype(np.float32)
        silent = (rng.standard_normal((4, 2)) * 2).astype(np.float32)
        shaped = np.stack([ref.haru_shape(x[r], cfg, np.array(HARU_IDS, np.int32), toks[:100 * (r + 1)], silent[r],
                                          *HARU_IDS, float(0.5 * r), r == 3) for r in range(4)])
        out[name] = dict(config=np.array(c[:3]), ints=np.array(c[3:], np.int32), tokens=toks, pen_tokens=pt,
                         pen_values=pv, counts=cnt, logits=x, silent=silent, shaped=shaped)
    return out


def main():
    build(ref=True)
    ref = RefSampler()
    q = qwen3_tts_cases(ref)
    np.savez_compressed(os.path.join(HERE, "qwen3_tts_cases.npz"),
                        **{f"{c}/{k}": v for c, d in q.items() for k, v in d.items()})
    lv = large_vocab_cases(ref)
    np.savez_compressed(os.path.join(HERE, "large_vocab_cases.npz"),
                        **{f"{c}/{k}": v for c, d in lv.items() for k, v in d.items()})
    h = haru_cases(ref)
    flat = {"logits": h.pop("logits")}
    flat.update({f"{c}/{k}": v for c, d in h.items() for k, v in d.items()})
    np.savez_compressed(os.path.join(HERE, "haru_cases.npz"), **flat)
    d = drama3_cases(ref)
    np.savez_compressed(os.path.join(HERE, "drama3_cases.npz"),
                        **{f"{c}/{k}": v for c, dd in d.items() for k, v in dd.items()})
    hd = haru_dry_cases(ref)
    np.savez_compressed(os.path.join(HERE, "haru_dry_cases.npz"),
                        **{f"{c}/{k}": v for c, dd in hd.items() for k, v in dd.items()})
    with open(os.path.join(HERE, "kat.json"), "w") as f:
        json.dump(kats(ref), f, indent=1)
    print("wrote", sorted(os.listdir(HERE)))


if __name__ == "__main__":
    main()
