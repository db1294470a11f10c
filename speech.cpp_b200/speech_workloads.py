"""Seeded synthetic inputs of the five benchmark configurations (no dataset or model is involved: the
sampler's inputs are logits rows, histories, masks and uniforms, generated here on the host with
numpy's PCG64 so the CPU checkers and the GPU engine see identical bytes).

config 1  greedy + suppress   fp32 [rows, 151936] N(0,1), one random index +8 per row, 64 banned ids
config 2  talker              fp32 [steps, 3072] N(0, 2^2); T 0.9, k 50, p 1, rep 1.05, 512-id history
config 3  code predictor      fp32 [64, 2048] N(0, 1.5^2) per step; T 0.9, k 50, p 1, no penalty
config 4  text decoder        bf16 [256, 151936] from fp32 N(0, 3^2) + Zipf offset; T 0.8, k 40, p 0.95,
                              presence 0.5, frequency 0.3, 1024 Zipf-distributed history ids per row
config 5  constrained         fp32 [B, 151936] N(0, 2^2), per-row allow mask of density d; T 1, k 0, p 0.9

Zipf offset (config 4): a seeded permutation `perm` of the vocabulary ranks the tokens; the token of
rank r gets logit offset -1.1 * ln(r + 1) (Zipf with s = 1.1), and history ids are drawn with
probability proportional to (r + 1)^-1.1 over the same ranking.
Uniforms: a seeded fp32 stream in [0, 1) (numpy random(dtype=float32)), promoted to double.
bf16: fp32 rounded to nearest even, stored as uint16 bit patterns.
"""
from __future__ import annotations

import numpy as np

QWEN3_VOCAB = 151936
TALKER_VOCAB = 3072
CP_VOCAB = 2048
ZIPF_S = 1.1


def to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 (round to nearest even), as uint16 bit patterns."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    r = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)
    return r


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32)


def pack_mask(bits: np.ndarray) -> np.ndarray:
    """bool [..., V] -> uint32 words [..., ceil(V/32)], bit (t & 31) of word t >> 5 = token t."""
    bits = np.asarray(bits, dtype=bool)
    v = bits.shape[-1]
    words = (v + 31) // 32
    padded = np.zeros(bits.shape[:-1] + (words * 32,), dtype=bool)
    padded[..., :v] = bits
    by = np.packbits(padded, axis=-1, bitorder="little")
    return np.ascontiguousarray(by).view(np.uint32)


def uniforms(seed: int, n: int) -> np.ndarray:
    return np.random.default_rng(seed).random(n, dtype=np.float32).astype(np.float64)


def config1(rows: int = 1000, vocab: int = QWEN3_VOCAB, seed: int = 1):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((rows, vocab), dtype=np.float32)
    hot = rng.integers(0, vocab, size=rows)
    x[np.arange(rows), hot] += np.float32(8.0)
    banned = np.zeros(vocab, bool)
    banned[rng.choice(vocab, size=64, replace=False)] = True
    return dict(logits=x, mask=pack_mask(banned), banned=banned, params=dict(greedy=True))


def config2(steps: int = 2048, vocab: int = TALKER_VOCAB, history: int = 512, seed: int = 2):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((steps, vocab), dtype=np.float32) * np.float32(2.0)
    h = rng.integers(0, vocab, size=(steps, history)).astype(np.int32)
    return dict(logits=x, history=h, u=uniforms(seed + 1000, steps),
                params=dict(temperature=0.9, top_k=50, top_p=1.0, repetition_penalty=1.05))


def config3(steps: int = 15, streams: int = 64, vocab: int = CP_VOCAB, seed: int = 3):
    """`steps` sequential [streams, vocab] steps (15 codebooks x frames in the full run)."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((steps, streams, vocab), dtype=np.float32) * np.float32(1.5)
    return dict(logits=x, u=uniforms(seed + 1000, steps * streams).reshape(steps, streams),
                params=dict(temperature=0.9, top_k=50, top_p=1.0))


def zipf_ranking(vocab: int, seed: int):
    rng = np.random.default_rng(seed)
    perm = rng.permutation(vocab)  # perm[r] = token of rank r
    offset = np.empty(vocab, np.float32)
    offset[perm] = (-ZIPF_S * np.log(np.arange(vocab, dtype=np.float64) + 1.0)).astype(np.float32)
    pmf = (np.arange(vocab, dtype=np.float64) + 1.0) ** -ZIPF_S
    cdf = np.cumsum(pmf / pmf.sum())
    return perm, offset, cdf


def config4(rows: int = 256, vocab: int = QWEN3_VOCAB, history: int = 1024, seed: int = 4, row0: int = 0):
    """Rows row0 .. row0+rows of the config-4 batch (each row has its own seed, so any shard of the
    256-row batch is generated identically wherever it is generated)."""
    perm, offset, cdf = zipf_ranking(vocab, seed)
    x = np.empty((rows, vocab), np.float32)
    h = np.empty((rows, history), np.int32)
    for i in range(rows):
        rr = np.random.default_rng([seed, row0 + i])
        x[i] = rr.standard_normal(vocab, dtype=np.float32) * np.float32(3.0) + offset
        ranks = np.searchsorted(cdf, rr.random(history), side="right")
        h[i] = perm[np.minimum(ranks, vocab - 1)]
    u = np.array([np.random.default_rng([seed, row0 + i, 7]).random(dtype=np.float32) for i in range(rows)],
                 np.float64)
    return dict(logits_bf16=to_bf16_bits(x), history=h, u=u,
                params=dict(temperature=0.8, top_k=40, top_p=0.95, presence_penalty=0.5, frequency_penalty=0.3))


def config5(rows: int = 64, density: float = 0.01, vocab: int = QWEN3_VOCAB, seed: int = 5, row0: int = 0):
    x = np.empty((rows, vocab), np.float32)
    allow = np.empty((rows, vocab), bool)
    for i in range(rows):
        rr = np.random.default_rng([seed, row0 + i])
        x[i] = rr.standard_normal(vocab, dtype=np.float32) * np.float32(2.0)
        allow[i] = np.random.default_rng([seed, row0 + i, int(density * 1e6)]).random(vocab) < density
    u = np.array([np.random.default_rng([seed, row0 + i, 7]).random(dtype=np.float32) for i in range(rows)],
                 np.float64)
    return dict(logits=x, mask=pack_mask(allow), allow=allow, u=u,
                params=dict(temperature=1.0, top_k=0, top_p=0.9))
