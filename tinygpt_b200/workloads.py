"""Seeded synthetic inputs for the five benchmark configurations.

All randomness comes from numpy.random.Generator(Philox(seed)); the GPU never
generates randomness, so the oracle and the CUDA path see identical inputs.
Shapes and distributions follow the reference's benchmark description:

  1 gpt2     V=50257  B=1     fp32 N(0,3^2), 5 ids +8; T=0.8 k=40 p=0.95; rep 1.1 / 128 uniform ids
  2 llama    V=32000  B=64    bf16 N(0,2.5^2) + Zipf(1.1) bias over a per-row permutation;
                              presence 0.5, frequency 0.3 / 1024 Zipf ids; T=0.7 p=0.9 min-p 0.05
  3 grammar  V=128256 B=256   fp32 N(0,3^2); 64 bitmasks of density U[2%,30%]; state U{0..63};
                              half greedy, half T=0.7 k=50
  4 serving  V=128256 B=2048  bf16 N(0,3^2) + Zipf bias; k~U{1..1024}, p~U[0.5,1], T~U[0.3,1.2];
                              rep 1.05 / 512 Zipf ids (the headline configuration)
  5 spec     V=128256 B=128 K=5 fp32 target N(0,3^2), draft = target + N(0,0.5^2); draft ids
                              drawn from softmax(draft/T); T=0.8

The Zipf bias gives the token of rank r (1-based, through the row's random
affine permutation r -> (a*r + c) mod V) the logit offset -1.1*ln(r); history
ids of configs 2 and 4 are Zipf(1.1) ranks mapped through the same permutation.
"""
from __future__ import annotations

import numpy as np

from ._lib import ROW_PARAMS_DTYPE

CONFIGS = {
    1: dict(name="gpt2-cpu", vocab=50257, batch=1, dtype="f32"),
    2: dict(name="llama-decode", vocab=32000, batch=64, dtype="bf16"),
    3: dict(name="grammar", vocab=128256, batch=256, dtype="f32"),
    4: dict(name="serving", vocab=128256, batch=2048, dtype="bf16"),
    5: dict(name="spec-verify", vocab=128256, batch=128, dtype="f32", K=5),
}


def rng(seed: int) -> np.random.Generator:
    return np.random.Generator(np.random.Philox(seed))


def to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit patterns (uint16), round to nearest even."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    r = u >> 16
    r &= 1
    r += np.uint32(0x7FFF)
    r += u
    r >>= 16
    return r.astype(np.uint16)


def bf16_bits_to_f32(h: np.ndarray) -> np.ndarray:
    return (h.astype(np.uint32) << 16).view(np.float32)


def pack_mask(bits: np.ndarray) -> np.ndarray:
    """bool [S, W*32] -> uint32 [S, W]; bit i of word w is token 32*w + i."""
    S, n = bits.shape
    return np.packbits(bits, axis=1, bitorder="little").view("<u4").reshape(S, n // 32).astype(np.uint32)


def _normal(g: np.random.Generator, sigma: float, shape) -> np.ndarray:
    x = g.standard_normal(size=shape, dtype=np.float32)
    x *= np.float32(sigma)
    return x


def _zipf_ranks(g: np.random.Generator, shape, V: int) -> np.ndarray:
    z = g.zipf(1.1, size=shape)
    return (z - 1) % V


class _AffinePerm:
    """Per-row random permutation of the vocab, rank r -> token (a*r + c) mod V
    with gcd(a, V) = 1 (vectorisable, unlike a full shuffle of every row)."""

    def __init__(self, g: np.random.Generator, B: int, V: int):
        a = g.integers(1, max(V, 2), size=B, dtype=np.int64)
        for i in range(B):
            while np.gcd(a[i], V) != 1:
                a[i] = (a[i] + 1) % V or 1
        self.a, self.c, self.V = a, g.integers(0, V, size=B, dtype=np.int64), V
        self.ainv = np.array([pow(int(x), -1, V) if V > 1 else 0 for x in a], np.int64)

    def token(self, ranks: np.ndarray) -> np.ndarray:  # ranks [B, n] (0-based) -> token ids
        return ((self.a[:, None] * ranks + self.c[:, None]) % self.V).astype(np.int32)

    def rank_of_tokens(self) -> np.ndarray:  # [B, V] 0-based rank of every token
        v = np.arange(self.V, dtype=np.int64)[None, :]
        return ((v - self.c[:, None]) % self.V * self.ainv[:, None]) % self.V


def _zipf_bias(perm: _AffinePerm) -> np.ndarray:
    rank_bias = (-1.1 * np.log(np.arange(1, perm.V + 1, dtype=np.float64))).astype(np.float32)
    B, V = len(perm.a), perm.V
    out = np.empty((B, V), np.float32)
    v = np.arange(V, dtype=np.int64)[None, :]
    for i in range(0, B, 32):  # row chunks keep the int64 temporaries small
        c, ai = perm.c[i:i + 32, None], perm.ainv[i:i + 32, None]
        out[i:i + 32] = rank_bias[((v - c) % V * ai) % V]
    return out


def make(config: int, seed: int = 0, batch: int | None = None, vocab: int | None = None) -> dict:
    """Inputs of one configuration (optionally with a smaller batch / vocab for tests)."""
    c = dict(CONFIGS[config])
    B = batch if batch is not None else c["batch"]
    V = vocab if vocab is not None else c["vocab"]
    g = rng(seed * 1000 + config)
    out = dict(config=config, name=c["name"], vocab=V, batch=B)
    p = np.zeros(B, ROW_PARAMS_DTYPE)
    p["top_p"] = 1.0
    if config == 1:
        x = _normal(g, 3.0, (B, V))
        for b in range(B):
            x[b, g.choice(V, 5, replace=False)] += 8.0
        p["temperature"] = 0.8
        p["top_k"] = 40
        p["top_p"] = 0.95
        p["repetition_penalty"] = 1.1
        hist = g.integers(0, V, size=(B, 128), dtype=np.int32)
        out.update(logits=x, history=hist, history_len=np.full(B, 128, np.int32))
    elif config == 2:
        perm = _AffinePerm(g, B, V)
        x = _normal(g, 2.5, (B, V)) + _zipf_bias(perm)
        p["temperature"] = 0.7
        p["top_p"] = 0.9
        p["min_p"] = 0.05
        p["presence_penalty"] = 0.5
        p["frequency_penalty"] = 0.3
        hist = perm.token(_zipf_ranks(g, (B, 1024), V))
        out.update(logits=to_bf16_bits(x), history=hist, history_len=np.full(B, 1024, np.int32))
    elif config == 3:
        x = _normal(g, 3.0, (B, V))
        W = (V + 31) // 32
        dens = g.uniform(0.02, 0.30, size=64)
        bits = g.random((64, W * 32)) < dens[:, None]
        bits[:, V:] = False
        table = pack_mask(bits)
        state = g.integers(0, 64, size=B, dtype=np.int32)
        greedy = np.arange(B) % 2 == 0
        p["temperature"] = np.where(greedy, 0.0, 0.7)
        p["top_k"] = np.where(greedy, 0, 50)
        out.update(logits=x, mask_table=table, state_id=state)
    elif config == 4:
        perm = _AffinePerm(g, B, V)
        x = _normal(g, 3.0, (B, V)) + _zipf_bias(perm)
        p["top_k"] = g.integers(1, 1025, size=B)
        p["top_p"] = g.uniform(0.5, 1.0, size=B)
        p["temperature"] = g.uniform(0.3, 1.2, size=B)
        p["repetition_penalty"] = 1.05
        hist = perm.token(_zipf_ranks(g, (B, 512), V))
        out.update(logits=to_bf16_bits(x), history=hist, history_len=np.full(B, 512, np.int32))
    elif config == 5:
        K = c["K"]
        T = 0.8
        tgt = _normal(g, 3.0, (B, K + 1, V))
        drf = tgt[:, :K, :] + _normal(g, 0.5, (B, K, V))
        s = drf.astype(np.float64) / T
        s -= s.max(axis=2, keepdims=True)
        pr = np.exp(s)
        cdf = np.cumsum(pr, axis=2)
        u = g.random((B, K)) * cdf[:, :, -1]
        ids = np.empty((B, K), np.int32)
        for b in range(B):
            for k in range(K):
                ids[b, k] = min(int(np.searchsorted(cdf[b, k], u[b, k], side="right")), V - 1)
        out.update(target=tgt, draft=drf, draft_ids=ids, K=K,
                   temperature=np.full(B, T, np.float32),
                   u_accept=g.random((B, K), dtype=np.float32),
                   u_draw=g.random(B, dtype=np.float32))
        return out
    out["params"] = p
    out["uniforms"] = g.random(B, dtype=np.float32)
    return out


def bytes_per_row(config: int, vocab: int | None = None) -> int:
    """Algorithmic HBM bytes per row: logits read once + history ids + the row's mask."""
    c = CONFIGS[config]
    V = vocab or c["vocab"]
    if config == 1:
        return V * 4 + 128 * 4
    if config == 2:
        return V * 2 + 1024 * 4
    if config == 3:
        return V * 4 + ((V + 31) // 32) * 4
    if config == 4:
        return V * 2 + 512 * 4
    if config == 5:
        K = c["K"]
        return (2 * K + 1) * V * 4 + K * 4
    raise ValueError(config)
