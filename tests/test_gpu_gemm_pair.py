"""The CTA-pair int8 GEMM (tcgen05 cta_group::2, gemm_pair.cu) against the
oracle: the same int32 accumulators and dequantized f32 bits as the
single-CTA kernel (linalg/int8_test.go:10, linalg/kernel_test.go:99), on
shapes whose last 256-row tile leaves the odd CTA partly or wholly outside
M, N not a multiple of 256 and K not a multiple of the 128-byte K block; and
every epilogue the encoder and the SigLIP tower use (GeGLU, residual
reduce-add, bias, GELU-tanh, the outlier terms) through whole forwards with
the pair kernel forced on (IG_GEMM_PAIR=1)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _case(M, N, K, seed, pad=16):
    rng = np.random.default_rng(seed)
    lda = (K + pad - 1) // pad * pad
    A = np.zeros((M, lda), np.uint8)
    A[:, :K] = rng.integers(1, 256, size=(M, K))
    B = np.zeros((N, lda), np.int8)
    B[:, :K] = rng.integers(-127, 128, size=(N, K))
    sa = np.exp(rng.uniform(np.log(1e-3), np.log(1e-1), M)).astype(np.float32)
    sb = np.exp(rng.uniform(np.log(1e-3), np.log(1e-1), N)).astype(np.float32)
    zc = (128.0 * B[:, :K].astype(np.int64).sum(1)).astype(np.float32)
    return A, B, sa, sb, zc


def _dev(*arrs):
    return [torch.from_numpy(a).cuda() for a in arrs]


def _bits(a):
    return np.ascontiguousarray(a).view(np.uint32)


@pytest.mark.parametrize("M,N,K", [(1, 256, 32), (7, 384, 1152), (129, 300, 301), (256, 768, 1152),
                                   (300, 2304, 768), (383, 512, 640), (4097, 768, 1152)])
def test_pair_gemm_bitexact(igdev, oracle_lib, monkeypatch, M, N, K):
    from indecis_b200 import ops
    monkeypatch.setenv("IG_GEMM_PAIR", "1")
    A, B, sa, sb, zc = _case(M, N, K, seed=M * 5 + N + K)
    rows = np.unique(np.r_[0:min(M, 48), max(0, M - 48):M])
    acc_ref = oracle_lib.gemm_u8s8(np.ascontiguousarray(A[rows, :K]), np.ascontiguousarray(B[:, :K]))
    dA, dB, dsa, dsb, dzc = _dev(A, B, sa, sb, zc)
    acc = ops.gemm_u8s8(dA, dB, K=K, int32_out=True).cpu().numpy()
    assert np.array_equal(acc[rows], acc_ref)
    # every row: the exact integer product (float64 sums of products below 2^53 are exact)
    full = A[:, :K].astype(np.float64) @ B[:, :K].astype(np.float64).T
    assert np.array_equal(acc.astype(np.float64), full)
    C = ops.gemm_u8s8(dA, dB, K=K, sa=dsa, sb=dsb, zc=dzc).cpu().numpy()
    assert np.array_equal(_bits(C[rows]), _bits(oracle_lib.dequant(acc_ref, sa[rows], sb, zc)))
    old = np.random.default_rng(2).standard_normal((M, N)).astype(np.float32)
    dC = torch.from_numpy(old.copy()).cuda()
    ops.gemm_u8s8(dA, dB, K=K, sa=dsa, sb=dsb, zc=dzc, C=dC, accumulate=True)
    want = oracle_lib.dequant(acc_ref, sa[rows], sb, zc, C_old=old[rows])
    assert np.array_equal(_bits(dC.cpu().numpy()[rows]), _bits(want))


def test_pair_equals_single_cta(igdev, monkeypatch):
    """A C2 sweep shape at 16384 rows: the pair kernel and the single-CTA
    kernel give the same bits for every element."""
    from indecis_b200 import ops
    M, N, K = 16384, 768, 1152
    A, B, sa, sb, zc = _case(M, N, K, seed=11)
    dA, dB, dsa, dsb, dzc = _dev(A, B, sa, sb, zc)
    out = {}
    for mode in ("0", "1"):
        monkeypatch.setenv("IG_GEMM_PAIR", mode)
        out[mode] = (ops.gemm_u8s8(dA, dB, int32_out=True).cpu().numpy(),
                     ops.gemm_u8s8(dA, dB, sa=dsa, sb=dsb, zc=dzc).cpu().numpy())
    assert np.array_equal(out["0"][0], out["1"][0])
    assert np.array_equal(_bits(out["0"][1]), _bits(out["1"][1]))
    full = A.astype(np.float64) @ B.astype(np.float64).T
    assert np.array_equal(out["1"][0].astype(np.float64), full)


def test_pair_encoder_c4_layer_shape(igdev, oracle_lib, monkeypatch):
    """C4's layer shape (QKV 768 -> 2304, GeGLU Wi, residual Wo / WoMLP with
    K = 768 / 1152) through the pair kernel, bit-exact against the oracle."""
    import oracle
    from indecis_b200 import synthetic as S
    from indecis_b200.model import Config, Model
    monkeypatch.setenv("IG_GEMM_PAIR", "1")
    cfg = dict(S.C4)
    cfg.update(layers=2, vocab=4096)
    W = S.weights(cfg, seed=9, gamma_noise=0.1)
    om, gm = oracle.Model(cfg, W), Model.from_arrays(Config.from_dict(cfg), W)
    ids, offs = S.ids_varlen(12, 1, 300, cfg["vocab"], seed=43)
    assert np.array_equal(_bits(gm.EncodeTokens((ids, offs))), _bits(om.encode(ids, offs, mode=1, threads=8)))
    ro, do = om.encode(ids, offs, dump_layer=0, threads=8)
    rg, dg = gm.encode_dump((ids, offs), 0)
    for k in ("xq", "cq", "hq", "gq"):
        assert np.array_equal(dg[k], do[k]), k
    for k in ("qkv", "ctx", "x_attn", "x_mlp"):
        assert np.array_equal(_bits(dg[k]), _bits(do[k])), k
    gm.close()


def test_pair_siglip_tower(igdev, oracle_lib, monkeypatch):
    """The SigLIP epilogues (bias, GELU-tanh, outlier terms + residual)
    through the pair kernel at C5's layer shape, bit-exact."""
    import oracle
    from indecis_b200 import synthetic as S
    from indecis_b200.siglip import Vision, VisionConfig
    monkeypatch.setenv("IG_GEMM_PAIR", "1")
    cfg = dict(S.C5)
    cfg.update(layers=1)
    W = S.siglip_weights(cfg, seed=5)
    om, gm = oracle.SigLIP(cfg, W), Vision.from_arrays(VisionConfig.from_dict(cfg), W)
    px = S.pixels(2, cfg["image_size"], seed=6)
    pa, po, do = om.forward(px, dump_layer=0, threads=2)
    dg, pg = gm.dump(px, 0)
    for k in ("h1q", "h2q", "mq"):
        assert np.array_equal(dg[k], do[k]), k
    for k in ("qkv", "attn", "x_attn", "mlp", "x_mlp"):
        assert np.array_equal(_bits(dg[k]), _bits(do[k])), k
    assert np.array_equal(_bits(pg), _bits(po))
    gm.close()
