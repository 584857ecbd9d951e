"""The oracle's SigLIP pieces (oracle/siglip.cpp) against their definitions
and the reference's properties: GeluTanh's two forms (vec_simd.go:166,
fastmath.go:28), the blocked float32 product (gemm.go:65-240),
MatMul8Outliers (int8.go:281-349) and Forward's layer/pool contract
(siglip_test.go:258 TestForwardLayers). CPU only."""
import numpy as np
import pytest

import oracle
from indecis_b200 import synthetic as S


def _f64_gelu_tanh(x):
    x = x.astype(np.float64)
    with np.errstate(over="ignore"):
        return x / (1 + np.exp(-2 * 0.7978845608028654 * (x + 0.044715 * x ** 3)))


def test_gelu_tanh_forms():
    x = np.concatenate([np.linspace(-12, 12, 4001), [0.0, -0.0, 1e-30, -1e-30, 88.0, -88.0, 200.0, -200.0]])
    x = x.astype(np.float32)
    n = x.size - x.size % 8
    vec = oracle.gelu_tanh(x[:n])                       # all through the vector body
    tail = np.concatenate([oracle.gelu_tanh(x[i:i + 1]) for i in range(n)])  # V = 8, one value: scalar tail
    ref = _f64_gelu_tanh(x[:n])
    assert np.abs(vec - ref).max() < 2e-6 * max(1.0, np.abs(ref).max())
    assert np.abs(tail - ref).max() < 2e-6 * max(1.0, np.abs(ref).max())
    # Both forms are close to the function in relative terms where it is not tiny.
    big = np.abs(ref) > 1e-3
    assert (np.abs(vec - ref)[big] / np.abs(ref)[big]).max() < 5e-6
    assert (np.abs(tail - ref)[big] / np.abs(ref)[big]).max() < 5e-6
    # The tail of a call is exactly the scalar form.
    y = oracle.gelu_tanh(x[:13])
    assert np.array_equal(y[8:], np.concatenate([oracle.gelu_tanh(x[i:i + 1]) for i in range(8, 13)]))


def test_linear_f32_blocks():
    rng = np.random.default_rng(3)
    for K in (1, 17, 256, 257, 512, 700, 768):
        x = rng.standard_normal((5, K)).astype(np.float32)
        W = rng.standard_normal((7, K)).astype(np.float32)
        b = rng.standard_normal(7).astype(np.float32)
        got = oracle.linear_f32(x, W, b)
        ref = x.astype(np.float64) @ W.T.astype(np.float64) + b
        assert np.abs(got - ref).max() < 1e-4 * np.sqrt(K)
        # 256-deep blocks, each one chain from zero, added in order, then the bias.
        parts = [oracle.linear_f32(x[:, k:k + 256], W[:, k:k + 256]) for k in range(0, K, 256)]
        tot = parts[0]
        for p in parts[1:]:
            tot = (tot + p).astype(np.float32)
        assert np.array_equal(got, (tot + b).astype(np.float32))


def _pack(w):
    n, k = w.shape
    q = np.zeros((n, k), np.int8)
    scale = np.zeros(n, np.float32)
    cs = np.zeros(n, np.int32)
    zc = np.zeros(n, np.float32)
    oracle.lib().or_pack_b8(np.ascontiguousarray(w, np.float32), k, n, 1, q, scale, cs, zc)
    return q, scale, zc


def _outliers(a, q, scale, zc, ratio=6.0):
    import ctypes as C
    m, k = a.shape
    n = q.shape[0]
    c = np.zeros((m, n), np.float32)
    out = np.zeros(32, np.int32)
    cnt = C.c_int32()
    oracle.lib().or_matmul8_outliers(c, np.ascontiguousarray(a, np.float32), m, q, scale, zc, k, n, ratio, out,
                                     C.byref(cnt))
    return c, out[:cnt.value]


@pytest.mark.parametrize("nmassive", [0, 3, 40])
def test_matmul8_outliers(nmassive):
    rng = np.random.default_rng(nmassive)
    m, k, n = 20, (256 if nmassive < 32 else 2048), 48
    a = np.abs(rng.standard_normal((m, k))).astype(np.float32)
    big = rng.choice(k, size=nmassive, replace=False)
    a[:, big] *= np.float32(50.0) * (1 + np.arange(nmassive, dtype=np.float32) / 7)[None, :] if nmassive else 1
    q, scale, zc = _pack(rng.standard_normal((n, k)).astype(np.float32) * 0.02)
    c, out = _outliers(a, q, scale, zc)
    colmax = np.abs(a).max(0)
    mean = np.float32(0)
    for v in colmax:
        mean = np.float32(mean + v)
    mean = np.float32(mean / np.float32(k))
    cand = [j for j in range(k) if colmax[j] > np.float32(6.0) * mean]
    if len(cand) > 32:  # the reference's partial selection sort (int8.go:313-324)
        for i in range(32):
            best = i
            for x in range(i + 1, len(cand)):
                if colmax[cand[x]] > colmax[cand[best]]:
                    best = x
            cand[i], cand[best] = cand[best], cand[i]
        cand = cand[:32]
    assert list(out) == cand
    assert len(out) == min(nmassive, 32)
    # The int8 product of the rest, then the float32 terms in that order.
    rest = a.copy()
    rest[:, out] = 0
    base = np.zeros((m, n), np.float32)
    oracle.lib().or_matmul8(base, rest, m, q, scale, zc, k, n, 0)
    for j in out:
        w = (q[:, j].astype(np.float32) * scale).astype(np.float32)
        base = (base + (a[:, j:j + 1] * w[None, :]).astype(np.float32)).astype(np.float32)
    assert np.array_equal(c, base)
    # Outliers keep the small channels' resolution: closer to float than plain int8.
    exact = a.astype(np.float64) @ (q.astype(np.float64) * scale[:, None]).T
    plain = np.zeros((m, n), np.float32)
    oracle.lib().or_matmul8(plain, a, m, q, scale, zc, k, n, 0)
    if nmassive:
        assert np.abs(c - exact).max() < np.abs(plain - exact).max()


def test_forward_layers_contract():
    """TestForwardLayers (siglip_test.go:258-290): Forward(l, no pool) stops
    after l layers; Forward(l, pool) returns the same patches and Embed's
    vector; Forward(0) gives the final patch features."""
    cfg = S.siglip_tiny(layers=3)
    m = oracle.SigLIP(cfg, S.siglip_weights(cfg, seed=2))
    px = S.pixels(2, cfg["image_size"], seed=3)
    stopped, none = m.forward(px, layer=2, pooled=False)
    assert none is None
    captured, pooled = m.forward(px, layer=2)
    assert np.array_equal(stopped, captured)
    final, emb = m.forward(px)
    assert np.array_equal(pooled, emb)
    assert not np.array_equal(final, captured)
    with pytest.raises(ValueError, match="the tower has 3"):
        m.forward(px, layer=4)
    # Images are independent: a batch equals its images one by one.
    one = np.concatenate([m.forward(px[i:i + 1])[1] for i in range(2)])
    assert np.array_equal(one, emb)
