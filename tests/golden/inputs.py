"""Seeded synthetic inputs shared by the golden-fixture generator, the tests and bench.py.

Distributions follow the BASELINE configs: activations ~N(0,1) fp16, int4 codes ~U{0..15},
scales ~U[1e-3, 2e-2] fp16, zero points ~U{0..15}, router logits ~N(0,1) (+ a Zipf-like
per-expert bias for prefill: bias_e = -1.1 * ln(rank_e), rank a seeded permutation of 1..E).
Everything is drawn from numpy.random.Generator(PCG64(seed)) in a fixed order, so every
machine regenerates identical arrays.
"""
from __future__ import annotations

import numpy as np


def _codes(rng, shape):
    return rng.integers(0, 16, size=shape, dtype=np.int64).astype(np.uint8)


def dense_case(seed: int, M: int, N: int, K: int, group: int, asym: bool = True):
    """x (M,K) f16, codes (N,K) u8, scales (N,K/g) f16, zeros (N,K/g) u8 or None."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((M, K), dtype=np.float32).astype(np.float16)
    codes = _codes(rng, (N, K))
    scales = rng.uniform(1e-3, 2e-2, size=(N, K // group)).astype(np.float16)
    zeros = _codes(rng, (N, K // group)) if asym else None
    return x, codes, scales, zeros


def expert_weights(rng, E: int, N: int, K: int, group: int, asym: bool = True):
    codes = _codes(rng, (E, N, K))
    scales = rng.uniform(1e-3, 2e-2, size=(E, N, K // group)).astype(np.float16)
    zeros = _codes(rng, (E, N, K // group)) if asym else None
    return codes, scales, zeros


def routing(rng, T: int, E: int, top_k: int, zipf_bias: bool = False):
    """Router logits ~N(0,1) (+ bias) -> softmax -> top-k -> renormalised weights."""
    logits = rng.standard_normal((T, E), dtype=np.float32)
    if zipf_bias:
        rank = rng.permutation(E) + 1
        logits = logits + (-1.1 * np.log(rank.astype(np.float32)))[None, :]
    lg = logits - logits.max(axis=1, keepdims=True)
    p = np.exp(lg)
    p = p / p.sum(axis=1, keepdims=True)
    ids = np.argsort(-p, axis=1, kind="stable")[:, :top_k].astype(np.int32)
    w = np.take_along_axis(p, ids, axis=1)
    w = (w / w.sum(axis=1, keepdims=True)).astype(np.float32)
    return logits, ids, w


def moe_layer_case(seed: int, T: int, E: int, H: int, inter: int, top_k: int, group: int,
                   asym: bool = True, zipf_bias: bool = False):
    """x (T,H) f16; w13 codes (E,2I,H), s13, z13; w2 codes (E,H,I), s2, z2; topk ids/weights."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((T, H), dtype=np.float32).astype(np.float16)
    c13, s13, z13 = expert_weights(rng, E, 2 * inter, H, group, asym)
    c2, s2, z2 = expert_weights(rng, E, H, inter, group, asym)
    _, ids, w = routing(rng, T, E, top_k, zipf_bias)
    return dict(x=x, c13=c13, s13=s13, z13=z13, c2=c2, s2=s2, z2=z2, topk_ids=ids,
                topk_weights=w)


def random_topk(seed: int, T: int, E: int, top_k: int):
    """Distinct experts per token, uniformly random (the reference tests' routing)."""
    rng = np.random.default_rng(seed)
    return np.stack([rng.permutation(E)[:top_k] for _ in range(T)]).astype(np.int32)
