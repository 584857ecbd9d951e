"""Seeded synthetic models and inputs for the workloads the encoder is measured on.

The reference publishes no checkpoint at these shapes; its benchmarks and
tests use random-init weights and ids (the model weights ~ N(0, 0.02) with
unit norm gains, heads ~ N(0, 0.02) with zero bias as heads.go:29-48 does).
All generators are numpy PCG64 streams with fixed seeds, so every process
(tests, bench, CPU baseline) sees the same tensors.
"""
from __future__ import annotations

import numpy as np

# Model shapes (transformers config.json field meanings, internal/modernbert/model.go:25-49).
C1 = dict(vocab=16384, hidden=256, layers=6, heads=4, intermediate=384, norm_eps=1e-5, global_every=3,
          local_attention=128, global_theta=10000.0, local_theta=10000.0, pooling="mean")
C4 = dict(vocab=262144, hidden=768, layers=22, heads=12, intermediate=1152, norm_eps=1e-5, global_every=3,
          local_attention=128, global_theta=10000.0, local_theta=10000.0, pooling="mean")


def tiny(layers=2, hidden=128, heads=2, intermediate=192, vocab=512, **kw):
    """A small model with the C1 structure, for quick parity cases."""
    cfg = dict(C1)
    cfg.update(vocab=vocab, hidden=hidden, layers=layers, heads=heads, intermediate=intermediate)
    cfg.update(kw)
    return cfg


def weights(cfg: dict, seed: int = 42, std: float = 0.02, gamma_noise: float = 0.0) -> dict:
    """float32 weights in transformers layouts (internal/modernbert/model.go:179-234)."""
    rng = np.random.default_rng(seed)
    H, I, L, V = cfg["hidden"], cfg["intermediate"], cfg["layers"], cfg["vocab"]

    def normal(*shape):
        return (rng.standard_normal(shape, dtype=np.float32) * np.float32(std)).astype(np.float32)

    def gamma():
        g = np.ones(H, np.float32)
        if gamma_noise:
            g += rng.standard_normal(H, dtype=np.float32) * np.float32(gamma_noise)
        return g

    w = dict(emb=normal(V, H), emb_norm=gamma(), final_norm=gamma(), attn_norm=[], wqkv=[], wo=[], mlp_norm=[],
             wi=[], wo_mlp=[])
    for l in range(L):
        w["attn_norm"].append(None if l == 0 else gamma())
        w["wqkv"].append(normal(3 * H, H))
        w["wo"].append(normal(H, H))
        w["mlp_norm"].append(gamma())
        w["wi"].append(normal(2 * I, H))
        w["wo_mlp"].append(normal(H, I))
    return w


def ids_fixed(nseq: int, n: int, vocab: int, seed: int = 1, lo: int = 4):
    """nseq sequences of n ids uniform in [lo, vocab), concatenated, with offsets."""
    rng = np.random.default_rng(seed)
    ids = rng.integers(lo, vocab, size=nseq * n, dtype=np.int64).astype(np.int32)
    offs = np.arange(nseq + 1, dtype=np.int64) * n
    return ids, offs


def ids_varlen(nseq: int, lmin: int, lmax: int, vocab: int, seed: int = 3, lo: int = 4):
    """nseq sequences with lengths uniform in [lmin, lmax], unpadded."""
    rng = np.random.default_rng(seed)
    lens = rng.integers(lmin, lmax + 1, size=nseq)
    offs = np.concatenate([[0], np.cumsum(lens)]).astype(np.int64)
    ids = rng.integers(lo, vocab, size=int(offs[-1]), dtype=np.int64).astype(np.int32)
    return ids, offs


def heads(hidden: int, seed: int = 7, std: float = 0.02):
    """The C1 decision heads (heads.go:29-48): noul, choice(5), score(5 levels), spans(4 types)."""
    rng = np.random.default_rng(seed)
    spec = [("noul", "noul", 1), ("choice", "choice", 5), ("score", "score", 4), ("spans", "spans", 9)]
    out = []
    for name, kind, rows in spec:
        w = (rng.standard_normal((rows, hidden), dtype=np.float32) * np.float32(std)).astype(np.float32)
        out.append(dict(name=name, kind=kind, w=w, b=np.zeros(rows, np.float32)))
    return out
