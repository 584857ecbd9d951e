"""The oracle's float32 encoder (or_encode_f32: the reference without
SetInt8, infer.go:304-430 with attendBlocks, :590-650) against a float64
numpy transformer of the same weights: equal to float32 accuracy, with
sequences long enough for several key blocks (the blocked softmax's
rescaling) in global and local layers; and close to the int8 path
(TestEncodeInt8's cosine bound, internal/modernbert/infer_test.go). CPU
only."""
import numpy as np

import oracle
from indecis_b200 import synthetic as S


def _ln(x, g, eps):
    m = x.mean(-1, keepdims=True)
    v = ((x - m) ** 2).mean(-1, keepdims=True)
    return (x - m) / np.sqrt(v + eps) * g


def _gelu(x):
    from scipy.special import erf
    return 0.5 * x * (1 + erf(x / np.sqrt(2)))


def _rope(theta, D, n):
    inv = 1.0 / theta ** (np.arange(0, D, 2) / D)
    f = np.outer(np.arange(n), inv)
    return np.cos(f), np.sin(f)


def _f64_encode(cfg, W, ids, offs):
    H, nh, I = cfg["hidden"], cfg["heads"], cfg["intermediate"]
    D = H // nh
    out = []
    for s in range(len(offs) - 1):
        sid = ids[offs[s]:offs[s + 1]]
        n = len(sid)
        x = _ln(W["emb"][sid].astype(np.float64), W["emb_norm"], cfg["norm_eps"])
        for l in range(cfg["layers"]):
            glob = l % cfg["global_every"] == 0
            h = x if l == 0 else _ln(x, W["attn_norm"][l], cfg["norm_eps"])
            qkv = h @ W["wqkv"][l].T.astype(np.float64)
            c, sn = _rope(cfg["global_theta"] if glob else cfg["local_theta"], D, n)
            ctx = np.zeros((n, H))
            for hh in range(nh):
                q, k, v = (qkv[:, j * H + hh * D:j * H + (hh + 1) * D] for j in range(3))
                rot = lambda a: np.concatenate([a[:, :D // 2] * c - a[:, D // 2:] * sn,
                                                a[:, D // 2:] * c + a[:, :D // 2] * sn], 1)
                q, k = rot(q), rot(k)
                sc = q @ k.T / np.sqrt(D)
                if not glob:
                    w = cfg["local_attention"] // 2
                    ii = np.arange(n)
                    sc[np.abs(ii[:, None] - ii[None, :]) > w] = -np.inf
                p = np.exp(sc - sc.max(1, keepdims=True))
                p /= p.sum(1, keepdims=True)
                ctx[:, hh * D:(hh + 1) * D] = p @ v
            x = x + ctx @ W["wo"][l].T
            z = _ln(x, W["mlp_norm"][l], cfg["norm_eps"]) @ W["wi"][l].T
            x = x + (_gelu(z[:, :I]) * z[:, I:]) @ W["wo_mlp"][l].T
        out.append(_ln(x, W["final_norm"], cfg["norm_eps"]).mean(0))
    return np.stack(out)


def test_f32_path_matches_float64():
    cfg = S.tiny(layers=3, hidden=128, heads=2, intermediate=192, vocab=400)
    W = S.weights(cfg, seed=8, gamma_noise=0.1)
    om = oracle.Model(cfg, W)
    ids, offs = S.ids_varlen(5, 1, 330, cfg["vocab"], seed=2, lo=0)  # up to three key blocks of 128
    got = om.encode_f32(ids, offs, threads=4)
    want = _f64_encode(cfg, W, ids, offs)
    assert np.abs(got - want).max() < 2e-5 * max(1.0, np.abs(want).max())


def test_f32_tokens_and_cls():
    cfg = S.tiny(layers=2, hidden=128, heads=2, intermediate=192, vocab=300, pooling="cls")
    om = oracle.Model(cfg, S.weights(cfg, seed=9))
    ids, offs = S.ids_varlen(4, 1, 140, cfg["vocab"], seed=5, lo=0)
    tok = om.encode_f32(ids, offs, mode=1)
    pooled = om.encode_f32(ids, offs, mode=0)
    assert np.array_equal(pooled, tok[offs[:-1]])


def test_int8_close_to_f32():
    """TestEncodeInt8: the int8 encoder stays close to float32 (cosine >= 0.99)."""
    cfg = S.tiny(layers=4, hidden=256, heads=4, intermediate=384, vocab=600)
    om = oracle.Model(cfg, S.weights(cfg, seed=10))
    ids, offs = S.ids_varlen(8, 4, 200, cfg["vocab"], seed=6)
    a, b = om.encode(ids, offs), om.encode_f32(ids, offs, threads=4)
    cos = (a * b).sum(1) / np.linalg.norm(a, axis=1) / np.linalg.norm(b, axis=1)
    assert cos.min() >= 0.99
