"""Row kernels vs the oracle, bit-exact: LayerNormRow (linalg/vec_simd.go:281),
quantizeA (linalg/int8.go:157; quant_amd64_test.go:11 TestQuantAVX2) and
PackB8 (linalg/int8.go:36)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("H", [1, 7, 16, 37, 64, 128, 256, 384, 768, 1153])
def test_layernorm_quant_bitexact(igdev, oracle_lib, H):
    from indecis_b200 import ops
    rng = np.random.default_rng(H)
    M = 67
    x = (rng.standard_normal((M, H)) * 3 + rng.uniform(-2, 2, (M, 1))).astype(np.float32)
    x[3] = 0.0  # a zero row: variance 0
    gamma = (1 + 0.1 * rng.standard_normal(H)).astype(np.float32)
    xn_ref = oracle_lib.layernorm(x, gamma, 1e-5, 8)
    q_ref, s_ref = oracle_lib.quantize_a(xn_ref)
    xn, q, sa = ops.layernorm_quant(torch.from_numpy(x).cuda(), torch.from_numpy(gamma).cuda())
    assert np.array_equal(xn.cpu().numpy().view(np.uint32), xn_ref.view(np.uint32))
    assert np.array_equal(q.cpu().numpy(), q_ref)
    assert np.array_equal(sa.cpu().numpy().view(np.uint32), s_ref.view(np.uint32))


def test_layernorm_lanes_16(igdev, oracle_lib):
    """The lane count is a parameter (16: the reference on AVX-512 hosts)."""
    from indecis_b200 import ops
    rng = np.random.default_rng(5)
    x = rng.standard_normal((33, 256)).astype(np.float32)
    g = np.ones(256, np.float32)
    ref = oracle_lib.layernorm(x, g, 1e-5, 16)
    xn, _, _ = ops.layernorm_quant(torch.from_numpy(x).cuda(), torch.from_numpy(g).cuda(), simd_lanes=16)
    assert np.array_equal(xn.cpu().numpy().view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("K", [1, 32, 256, 301, 384, 768, 1024, 1152, 2048, 3072, 4096])
def test_quantize_rows_bitexact(igdev, oracle_lib, K):
    from indecis_b200 import ops
    rng = np.random.default_rng(K)
    x = (rng.standard_normal((50, K)) * rng.uniform(0.01, 10, (50, 1))).astype(np.float32)
    x[7] = 0.0
    x[9, :] = 0.5  # ties: x * (127/0.5) lands on exact halves only through rounding
    x[11] *= np.float32(1e-37)  # scale max/127 below the normal range: the clamped path
    x[12] *= np.float32(3e36)   # large but finite
    q_ref, s_ref = oracle_lib.quantize_a(x)
    q, sa = ops.quantize_rows(torch.from_numpy(x).cuda())
    assert np.array_equal(q.cpu().numpy(), q_ref)
    assert np.array_equal(sa.cpu().numpy().view(np.uint32), s_ref.view(np.uint32))


@pytest.mark.parametrize("n,k", [(768, 256), (256, 384), (17, 301), (1, 1)])
def test_pack_b8_bitexact(igdev, oracle_lib, n, k):
    from indecis_b200 import ops
    rng = np.random.default_rng(n + k)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    if n > 3:
        w[2] = 0.0
        w[3, :4] = [0.5, -0.5, 1.0, -1.0]  # half-away rounding cases after scaling
    q_ref, s_ref, cs_ref, zc_ref = oracle_lib.pack_b8(w)
    q, s, zc, cs = ops.pack_b8(torch.from_numpy(w).cuda())
    q = q.cpu().numpy()
    assert np.array_equal(q[:, :k], q_ref)
    assert not q[:, k:].any()
    assert np.array_equal(s.cpu().numpy().view(np.uint32), s_ref.view(np.uint32))
    assert np.array_equal(zc.cpu().numpy().view(np.uint32), zc_ref.view(np.uint32))
    assert np.array_equal(cs.cpu().numpy(), cs_ref)


@pytest.mark.parametrize("K", [1, 256, 384, 301])
def test_quantize_rows_nan_inf(igdev, oracle_lib, K):
    """NaN and out-of-range products convert as the reference's VCVTPS2DQ does
    (INT_MIN, saturated to -128); a row whose only non-zero values are NaN is
    a zero row (all 128)."""
    from indecis_b200 import ops
    rng = np.random.default_rng(K + 1)
    x = rng.standard_normal((8, K)).astype(np.float32)
    x[0, K // 2] = np.nan
    x[1, K - 1] = np.inf
    x[2, 0] = -np.inf
    x[3, :] = np.nan
    x[4, :] = 0.0
    x[4, K // 3] = np.nan
    x[5, 0] = np.nan
    x[5] *= np.float32(1e-37)
    q_ref, s_ref = oracle_lib.quantize_a(x)
    q, sa = ops.quantize_rows(torch.from_numpy(x).cuda())
    assert np.array_equal(q.cpu().numpy(), q_ref)
    assert np.array_equal(sa.cpu().numpy().view(np.uint32), s_ref.view(np.uint32))


@pytest.mark.parametrize("H", [128, 256, 384])
def test_layernorm_quant_nan_gamma(igdev, oracle_lib, H):
    """A NaN in gamma makes that output NaN; the quantized row follows the
    reference's conversion for it and its NaN-ignoring maximum."""
    from indecis_b200 import ops
    rng = np.random.default_rng(H + 3)
    x = rng.standard_normal((9, H)).astype(np.float32)
    gamma = (1 + 0.1 * rng.standard_normal(H)).astype(np.float32)
    gamma[H // 5] = np.nan
    xn_ref = oracle_lib.layernorm(x, gamma, 1e-5, 8)
    q_ref, s_ref = oracle_lib.quantize_a(xn_ref)
    xn, q, sa = ops.layernorm_quant(torch.from_numpy(x).cuda(), torch.from_numpy(gamma).cuda())
    got = xn.cpu().numpy()
    assert np.array_equal(np.isnan(got), np.isnan(xn_ref))
    ok = ~np.isnan(xn_ref)
    assert np.array_equal(got[ok].view(np.uint32), xn_ref[ok].view(np.uint32))
    assert np.array_equal(q.cpu().numpy(), q_ref)
    assert np.array_equal(sa.cpu().numpy().view(np.uint32), s_ref.view(np.uint32))


def test_layernorm_quant_many_rows(igdev, oracle_lib):
    """Enough rows (H = 256) that every CTA of the staged LayerNorm kernel
    (the f32-output norm) walks several row groups and reuses each
    shared-memory stage; zero rows, NaN rows, huge rows and a ragged last group
    among them. The quantizing kernel runs on the same rows."""
    from indecis_b200 import ops
    rng = np.random.default_rng(77)
    M, H = 40003, 256
    x = (rng.standard_normal((M, H)) * 2 + rng.uniform(-3, 3, (M, 1))).astype(np.float32)
    x[5] = 0.0
    x[1000, 17] = np.nan
    x[30000] *= 1e30
    x[M - 1] = 1e-30
    gamma = (1 + 0.1 * rng.standard_normal(H)).astype(np.float32)
    xn_ref = oracle_lib.layernorm(x, gamma, 1e-5, 8)
    q_ref, s_ref = oracle_lib.quantize_a(xn_ref)
    dx, dg = torch.from_numpy(x).cuda(), torch.from_numpy(gamma).cuda()
    xn, q, sa = ops.layernorm_quant(dx, dg)
    xn_only, _, _ = ops.layernorm_quant(dx, dg, want_q=False)  # the staged kernel (f32 output only)
    assert np.array_equal(xn_only.cpu().numpy().view(np.uint32), xn.cpu().numpy().view(np.uint32))
    got = xn.cpu().numpy()
    assert np.array_equal(np.isnan(got), np.isnan(xn_ref)) and np.isnan(xn_ref[1000]).all()
    ok = ~np.isnan(xn_ref)
    assert np.array_equal(got[ok].view(np.uint32), xn_ref[ok].view(np.uint32))
    assert np.array_equal(q.cpu().numpy(), q_ref)
    assert np.array_equal(sa.cpu().numpy().view(np.uint32), s_ref.view(np.uint32))
