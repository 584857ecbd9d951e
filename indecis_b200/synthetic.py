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


# ---- SigLIP vision tower (internal/siglip; transformers SiglipVisionConfig) ----
# C5: ViT-B/16 at 224 px: 196 patches, hidden 768, 12 layers, 12 heads, MLP 3072.
C5 = dict(hidden=768, layers=12, heads=12, mlp=3072, image_size=224, patch_size=16, eps=1e-6)


def siglip_tiny(layers=2, hidden=128, heads=2, mlp=256, image_size=32, patch_size=8, **kw):
    """A small tower with C5's structure (16 patches), for quick parity cases."""
    cfg = dict(hidden=hidden, layers=layers, heads=heads, mlp=mlp, image_size=image_size, patch_size=patch_size,
               eps=1e-6)
    cfg.update(kw)
    return cfg


def siglip_weights(cfg: dict, seed: int = 42, std: float = 0.02, massive: int = 4, massive_gain: float = 20.0):
    """float32 tower weights, N(0, std) matrices and biases, norm gains near 1.

    `massive` fc1 channels per layer get `massive_gain` times larger weights
    and a positive bias: their GELU outputs reach tens while the others stay
    near one — the "massive activations" of trained vision transformers that
    MatMul8Outliers (linalg/int8.go:281) takes out of the int8 product.
    """
    rng = np.random.default_rng(seed)
    H, M, L, P = cfg["hidden"], cfg["mlp"], cfg["layers"], cfg["patch_size"]
    T = (cfg["image_size"] // P) ** 2

    def normal(*shape, s=std):
        return (rng.standard_normal(shape, dtype=np.float32) * np.float32(s)).astype(np.float32)

    def gain():
        return (1 + rng.standard_normal(H, dtype=np.float32) * np.float32(0.1)).astype(np.float32)

    w = dict(patch_w=normal(H, 3 * P * P), patch_b=normal(H), pos=normal(T, H), post_g=gain(), post_b=normal(H),
             probe=normal(H, s=1.0), in_w=normal(3 * H, H), in_b=normal(3 * H), hout_w=normal(H, H), hout_b=normal(H),
             hln_g=gain(), hln_b=normal(H), hfc1_w=normal(M, H), hfc1_b=normal(M), hfc2_w=normal(H, M),
             hfc2_b=normal(H))
    for k in ("ln1_g", "ln1_b", "ln2_g", "ln2_b", "wqkv", "bqkv", "wo", "bo", "w1", "b1", "w2", "b2"):
        w[k] = []
    for _ in range(L):
        w["ln1_g"].append(gain()), w["ln1_b"].append(normal(H))
        w["ln2_g"].append(gain()), w["ln2_b"].append(normal(H))
        w["wqkv"].append(normal(3 * H, H)), w["bqkv"].append(normal(3 * H))
        w["wo"].append(normal(H, H)), w["bo"].append(normal(H))
        w1, b1 = normal(M, H), normal(M)
        if massive:
            ch = rng.choice(M, size=massive, replace=False)
            w1[ch] *= np.float32(massive_gain)
            b1[ch] += np.float32(2.0)
        w["w1"].append(w1), w["b1"].append(b1)
        w["w2"].append(normal(H, M)), w["b2"].append(normal(H))
    return w


def pixels(n: int, image_size: int, seed: int = 5):
    """n images of normalized pixels [n][3][S][S], uniform in [-1, 1]."""
    rng = np.random.default_rng(seed)
    return rng.uniform(-1.0, 1.0, size=(n, 3, image_size, image_size)).astype(np.float32)
