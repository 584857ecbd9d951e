"""Pins the CPU oracle to the reference's own known-answer data and
exactness/accuracy properties (the reference cannot run here and ships no
int8 golden vectors; see oracle/oracle.h). Each test names the reference
test it restates."""
import math
import struct

import numpy as np
import pytest


def f32_bits(v):
    return struct.unpack("<I", struct.pack("<f", v))[0]


def test_round_half_even_kat(oracle_lib):
    """linalg/int8_test.go:88-94 TestRoundHalfEven: the listed values."""
    for v in [0, 0.5, 1.5, 2.5, -0.5, -1.5, 126.7, -127, 3.49999, -3.5000002]:
        v = float(np.float32(v))
        assert oracle_lib.round_half_even(v) == float(np.float32(round(v)))  # Python round: half to even


def test_gelu_constants_match_assembly(oracle_lib):
    """The float32 constants of the GeluMul restatement are the DATA words of
    linalg/gelu_amd64.s (geluRs2 .. geluB0)."""
    words = {"rs2": 0x3f3504f3, "a13": 0xaf95df0b, "a11": 0x32edffee, "a9": 0xb60cff51, "a7": 0xb86ec2d2,
             "half": 0x3f000000, "one": 0x3f800000, "lo": 0xc0800000, "hi": 0x40800000}
    vals = {"rs2": 0.7071067811865476, "a13": -2.72614225801306e-10, "a11": 2.77068142495902e-08,
            "a9": -2.10102402082508e-06, "a7": -5.69250639462346e-05, "half": 0.5, "one": 1.0, "lo": -4.0,
            "hi": 4.0}
    for k, w in words.items():
        assert f32_bits(vals[k]) == w, k


def test_exp32_accuracy(oracle_lib):
    """fastmath.go:35 exp32 (Cephes, relative error ~2e-7) and 0 below -87.3."""
    xs = np.linspace(-87, 88, 20001, dtype=np.float32)
    for x in xs[::37]:
        e = oracle_lib.lib().or_exp32(float(x))
        ref = math.exp(float(x))
        assert abs(e - ref) <= 4e-7 * ref, x
    assert oracle_lib.lib().or_exp32(-87.31) == 0.0


def test_exp_shift_body_and_tail(oracle_lib):
    """vec_simd.go:216-264: body (FMA) and tail (exp32) both within Cephes
    accuracy; the split depends on the position (n mod V)."""
    rng = np.random.default_rng(0)
    for n in (1, 7, 8, 9, 37, 129):
        x = rng.uniform(-20, 0, n).astype(np.float32)
        e, s = oracle_lib.exp_shift(x, 0.0, 8)
        assert np.allclose(e, np.exp(x.astype(np.float64)), rtol=5e-7, atol=0)
        assert abs(s - e.astype(np.float64).sum()) <= 1e-5 * e.sum()


@pytest.mark.parametrize("V", [1, 16, 32])
def test_lane_widths(oracle_lib, V):
    """The lane chains at every width a config may name (simd_lanes 1..32):
    ExpShift's body sums lane by lane, LayerNorm's mean and variance too;
    each stays within float32 accuracy of float64."""
    rng = np.random.default_rng(V)
    for n in (V - 1 if V > 1 else 1, 2 * V + 5, 129):
        x = rng.uniform(-20, 0, n).astype(np.float32)
        e, s = oracle_lib.exp_shift(x, 0.0, V)
        assert np.allclose(e, np.exp(x.astype(np.float64)), rtol=5e-7, atol=0)
        assert abs(s - e.astype(np.float64).sum()) <= 1e-5 * e.sum()
        xr = rng.standard_normal((3, n)).astype(np.float32)
        o = oracle_lib.layernorm(xr, np.ones(n, np.float32), V=V)
        d = xr.astype(np.float64)
        want = (d - d.mean(1, keepdims=True)) / np.sqrt(d.var(1, keepdims=True) + 1e-5)
        assert np.abs(o - want).max() <= 1e-4


@pytest.mark.parametrize("n", [1, 7, 16, 37, 384, 1153])
def test_vector_ops(oracle_lib, n):
    """linalg/vec_test.go:9 TestVectorOps: AbsMax exact, QuantizeRow exact,
    GeluMul within 1e-5 of the erf GELU."""
    rng = np.random.default_rng(1)
    x = (rng.standard_normal(n) * 3).astype(np.float32)
    b = rng.standard_normal(n).astype(np.float32)
    q, s = oracle_lib.quantize_a(x[None, :])
    want_max = np.abs(x).max()
    assert s[0] == np.float32(want_max) / np.float32(127)
    inv = np.float32(1) / s[0]
    want_q = (np.rint(x * inv).astype(np.int32) + 128).astype(np.uint8)
    assert np.array_equal(q[0], want_q)
    o = oracle_lib.gelu_mul(x, b)
    xd = x.astype(np.float64)
    g = 0.5 * xd * (1 + np.vectorize(math.erf)(xd / math.sqrt(2))) * b
    assert np.all(np.abs(o - g) <= 1e-5 * (1 + np.abs(g)))


def test_gelu_tails(oracle_lib):
    """quant_amd64_test.go:94 TestGeluMulAVX2: tails up to +-50."""
    x = np.linspace(-50, 50, 1601, dtype=np.float32)
    o = oracle_lib.gelu_mul(x, np.ones_like(x))
    xd = x.astype(np.float64)
    g = 0.5 * xd * (1 + np.vectorize(math.erf)(xd / math.sqrt(2)))
    assert np.all(np.abs(o - g) <= 1e-5 * (1 + np.abs(g)))


@pytest.mark.parametrize("m,k,n", [(1, 1, 1), (7, 384, 1152), (15, 1152, 384), (33, 301, 17)])
def test_matmul8_accuracy(oracle_lib, m, k, n):
    """linalg/int8_test.go:36 TestMatMul8: relative error <= 0.02 vs float,
    accumulate doubles within 1e-4."""
    rng = np.random.default_rng(2)
    a = rng.standard_normal((m, k)).astype(np.float32)
    w = rng.standard_normal((n, k)).astype(np.float32)
    q, s, cs, zc = oracle_lib.pack_b8(w)
    got = oracle_lib.matmul8(a, q, s, zc)
    want = a.astype(np.float64) @ w.astype(np.float64).T
    rel = np.sqrt(((got - want) ** 2).sum() / (want ** 2).sum())
    assert rel <= 0.02
    twice = oracle_lib.matmul8(a, q, s, zc, c_old=got)
    assert np.all(np.abs(twice - 2 * got) <= 1e-4 * np.abs(got) + 1e-6)


def test_pack_b8_half_away(oracle_lib):
    """linalg/int8.go:67: weights round half away from zero (math.Round)."""
    w = np.array([[127.0, 0.5, -0.5, 1.5, -1.5, 2.5]], np.float32)
    q, s, cs, zc = oracle_lib.pack_b8(w)
    assert s[0] == 1.0
    assert list(q[0]) == [127, 1, -1, 2, -2, 3]
    assert cs[0] == 130 and zc[0] == 128 * 130


def test_matmul8_rows_independent(oracle_lib):
    """linalg/int8_test.go:149 TestMatMul8RowsIndependent."""
    rng = np.random.default_rng(3)
    a = rng.standard_normal((13, 70)).astype(np.float32)
    w = rng.standard_normal((40, 70)).astype(np.float32)
    q, s, cs, zc = oracle_lib.pack_b8(w)
    full = oracle_lib.matmul8(a, q, s, zc)
    for i in range(13):
        assert np.array_equal(oracle_lib.matmul8(a[i:i + 1], q, s, zc)[0], full[i])


def _attend_ref(q, k, v, window):
    n, D = q.shape
    s = q.astype(np.float64) @ k.astype(np.float64).T / math.sqrt(D)
    if window >= 0:
        i = np.arange(n)
        s[np.abs(i[:, None] - i[None, :]) > window] = -np.inf
    p = np.exp(s - s.max(1, keepdims=True))
    return (p / p.sum(1, keepdims=True)) @ v.astype(np.float64)


@pytest.mark.parametrize("D", [64, 32])
@pytest.mark.parametrize("n", [1, 5, 17, 48, 100, 259])
@pytest.mark.parametrize("window", [-1, 8, 64])
def test_attend8_accuracy(oracle_lib, D, n, window):
    """linalg/attention8_test.go:50 TestAttend8: rel <= 0.03, worst <= 0.25,
    every output written (NaN prefill)."""
    rng = np.random.default_rng(n * 100 + D + window)
    q = (rng.standard_normal((n, D)) * 2).astype(np.float32)
    k = (rng.standard_normal((n, D)) * 2 + (np.arange(n * D) % D % 7).reshape(n, D)).astype(np.float32)
    v = rng.standard_normal((n, D)).astype(np.float32)
    o = oracle_lib.attn8(q, k, v, window, np.float32(1 / math.sqrt(D)))
    assert not np.isnan(o).any()
    want = _attend_ref(q, k, v, window)
    d = o - want
    rel = math.sqrt((d ** 2).sum() / max((want ** 2).sum(), 1e-30))
    assert rel <= 0.03 and np.abs(d).max() <= 0.25


def test_attn8_internals(oracle_lib):
    """Attn8 invariants: quantized P sums to 1/sp; K centred per the mean;
    scores from the integer accumulators ((acc - kzc) * ks) * sq."""
    rng = np.random.default_rng(4)
    n, D = 70, 64
    q, k, v = (rng.standard_normal((n, D)).astype(np.float32) for _ in range(3))
    o, dbg = oracle_lib.attn8(q, k, v, 8, np.float32(0.125), debug=True)
    for i in range(n):
        assert np.float32(1) / np.float32(dbg["p"][i].astype(np.int64).sum()) == dbg["sp"][i]
        assert dbg["p"][i].max() == 255
    acc = dbg["qa"].astype(np.int64) @ dbg["kq"].astype(np.int64).T
    mask = np.abs(np.arange(n)[:, None] - np.arange(n)[None, :]) <= 8
    assert np.array_equal(dbg["sacc"][mask], acc[mask])
    assert np.array_equal(dbg["kzc"], (128 * dbg["kq"].astype(np.int64).sum(1)).astype(np.float32))


def _float_forward(cfg, W, ids, offs):
    """Float64 ModernBERT forward (no quantization) for the int8 accuracy pin."""
    H, nh, I = cfg["hidden"], cfg["heads"], cfg["intermediate"]
    D = H // nh
    def ln(x, g):
        m = x.mean(1, keepdims=True)
        return (x - m) / np.sqrt(((x - m) ** 2).mean(1, keepdims=True) + cfg["norm_eps"]) * g
    x = ln(W["emb"][ids].astype(np.float64), W["emb_norm"])
    pos = np.concatenate([np.arange(offs[i + 1] - offs[i]) for i in range(len(offs) - 1)])
    inv = 1.0 / cfg["global_theta"] ** (np.arange(0, D, 2) / D)
    ang = pos[:, None] * inv[None, :]
    c, s = np.cos(ang), np.sin(ang)
    for l in range(cfg["layers"]):
        h = x if l == 0 else ln(x, W["attn_norm"][l])
        qkv = h @ W["wqkv"][l].T
        out = np.zeros((len(ids), H))
        for hh in range(nh):
            q = qkv[:, hh * D:(hh + 1) * D]
            k = qkv[:, H + hh * D:H + (hh + 1) * D]
            v = qkv[:, 2 * H + hh * D:2 * H + (hh + 1) * D]
            rot = lambda t: np.concatenate([t[:, :D // 2] * c - t[:, D // 2:] * s, t[:, D // 2:] * c + t[:, :D // 2] * s], 1)
            q, k = rot(q), rot(k)
            for b in range(len(offs) - 1):
                a, e = offs[b], offs[b + 1]
                w = -1 if l % cfg["global_every"] == 0 else cfg["local_attention"] // 2
                out[a:e, hh * D:(hh + 1) * D] = _attend_ref(q[a:e], k[a:e], v[a:e], w)
        x = x + out @ W["wo"][l].T
        h = ln(x, W["mlp_norm"][l])
        z = h @ W["wi"][l].T
        g = 0.5 * z[:, :I] * (1 + np.vectorize(math.erf)(z[:, :I] / math.sqrt(2))) * z[:, I:]
        x = x + g @ W["wo_mlp"][l].T
    x = ln(x, W["final_norm"])
    return np.stack([x[offs[i]:offs[i + 1]].mean(0) for i in range(len(offs) - 1)])


def test_encoder_int8_close_to_float(oracle_lib):
    """internal/modernbert/infer_test.go:195 TestEncodeInt8: cosine >= 0.99
    between the int8 and float encodings (random weights here)."""
    import oracle
    from indecis_b200 import synthetic as S
    cfg = S.tiny(layers=3, hidden=128, heads=2, intermediate=192, vocab=500)
    W = S.weights(cfg, std=0.05)
    ids, offs = S.ids_varlen(5, 8, 150, cfg["vocab"], seed=2)
    got = oracle.Model(cfg, W).encode(ids, offs)
    want = _float_forward(cfg, W, ids, offs)
    for a, b in zip(got, want):
        assert np.dot(a, b) / np.linalg.norm(a) / np.linalg.norm(b) >= 0.99


def test_cpu_baseline_bitexact(oracle_lib):
    """The timed CPU baseline (VNNI tiles, threads) equals the scalar oracle
    bit for bit (linalg/int8_test.go:10 TestMicroKernel8MatchesGo at model level)."""
    import oracle
    from indecis_b200 import synthetic as S
    cfg = S.tiny(layers=2, hidden=256, heads=4, intermediate=384, vocab=700)
    m = oracle.Model(cfg, S.weights(cfg))
    ids, offs = S.ids_varlen(11, 1, 220, cfg["vocab"], seed=4)
    a = m.encode(ids, offs)
    b = m.encode(ids, offs, threads=4, fast=True)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    t1 = m.encode(ids, offs, mode=1)
    t2 = m.encode(ids, offs, mode=1, threads=3)
    assert np.array_equal(t1.view(np.uint32), t2.view(np.uint32))


@pytest.mark.parametrize("case", ["d32_windows", "ragged_widths", "extreme"])
def test_cpu_baseline_vector_forms_bitexact(oracle_lib, case):
    """The CPU baseline's AVX2 / VNNI forms (LayerNorm lanes, row quantization,
    ExpShift, GeluMul, RoPE, attention tiles) equal the scalar loops bit for
    bit: head dimension 32 with local windows over long sequences, widths that
    leave scalar tails (hidden 200, intermediate 100, D = 50: the vector
    attention declines and the scalar one runs), and weights large enough to
    overflow to infinity (the rows with non-finite values take the scalar
    form)."""
    import oracle
    from indecis_b200 import synthetic as S
    if case == "d32_windows":
        cfg = S.tiny(layers=3, hidden=128, heads=4, intermediate=192, vocab=300)
        ids, offs = S.ids_varlen(6, 1, 400, cfg["vocab"], seed=8)
        W = S.weights(cfg)
    elif case == "ragged_widths":
        cfg = S.tiny(layers=2, hidden=200, heads=4, intermediate=100, vocab=300)
        ids, offs = S.ids_varlen(5, 1, 170, cfg["vocab"], seed=9)
        W = S.weights(cfg)
    else:
        cfg = S.tiny(layers=2, hidden=128, heads=2, intermediate=192, vocab=300)
        ids, offs = S.ids_varlen(4, 3, 140, cfg["vocab"], seed=10)
        W = S.weights(cfg)
        W["wqkv"][1] = (W["wqkv"][1] * np.float32(1e37)).astype(np.float32)
        W["wi"][0] = (W["wi"][0] * np.float32(1e36)).astype(np.float32)
        W["wo"][0][:5] = 0.0
    m = oracle.Model(cfg, W)
    for mode in (0, 1):
        a = m.encode(ids, offs, mode=mode)
        b = m.encode(ids, offs, mode=mode, threads=3, fast=True)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), mode


def test_out_of_vocabulary(oracle_lib):
    import oracle
    from indecis_b200 import synthetic as S
    cfg = S.tiny(layers=1, vocab=50)
    m = oracle.Model(cfg, S.weights(cfg))
    with pytest.raises(ValueError, match="id 50 out of vocabulary"):
        m.encode(np.array([1, 50], np.int32), np.array([0, 2], np.int64))


def test_encode_rejects_inconsistent_offsets(oracle_lib):
    """infer.go:245-247: offsets must start at 0 and never decrease."""
    import oracle
    from indecis_b200 import synthetic as S
    cfg = S.tiny(layers=1, hidden=64, heads=2, intermediate=96, vocab=100)
    om = oracle.Model(cfg, S.weights(cfg))
    ids = np.arange(10, dtype=np.int32)
    for offs in ([0, 6, 4, 10], [1, 5, 10]):
        with pytest.raises(ValueError, match="inconsistent"):
            om.encode(ids, np.asarray(offs, np.int64))
