"""tcgen05 int8 GEMM vs the oracle: int32 accumulators and dequantized f32
bit-exact (linalg/int8_test.go:10 TestMicroKernel8MatchesGo,
linalg/kernel_test.go:99 TestMicroKernel8DeqMatchesDequantize), rows
independent of their batch (int8_test.go:149), and the C2 sweep shapes."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _case(M, N, K, seed, pad=16):
    rng = np.random.default_rng(seed)
    lda = (K + pad - 1) // pad * pad
    A = np.zeros((M, lda), np.uint8)
    A[:, :K] = rng.integers(1, 256, size=(M, K))  # q + 128, q in [-127, 127]
    B = np.zeros((N, lda), np.int8)
    B[:, :K] = rng.integers(-127, 128, size=(N, K))
    sa = np.exp(rng.uniform(np.log(1e-3), np.log(1e-1), M)).astype(np.float32)
    sb = np.exp(rng.uniform(np.log(1e-3), np.log(1e-1), N)).astype(np.float32)
    zc = (128.0 * B[:, :K].astype(np.int64).sum(1)).astype(np.float32)
    return A, B, sa, sb, zc


def _dev(*arrs):
    return [torch.from_numpy(a).cuda() for a in arrs]


@pytest.mark.parametrize("M,N,K", [(1, 16, 32), (7, 384, 1152), (15, 1152, 384), (33, 17, 301), (128, 768, 256),
                                   (300, 256, 384), (129, 2304, 768), (256, 768, 1152), (5, 40, 70)])
def test_gemm_int32_and_f32_bitexact(igdev, oracle_lib, M, N, K):
    from indecis_b200 import ops
    A, B, sa, sb, zc = _case(M, N, K, seed=M * 7 + N)
    acc_ref = oracle_lib.gemm_u8s8(np.ascontiguousarray(A[:, :K]), np.ascontiguousarray(B[:, :K]))
    dA, dB, dsa, dsb, dzc = _dev(A, B, sa, sb, zc)
    acc = ops.gemm_u8s8(dA, dB, K=K, int32_out=True).cpu().numpy()
    assert np.array_equal(acc, acc_ref)
    C = ops.gemm_u8s8(dA, dB, K=K, sa=dsa, sb=dsb, zc=dzc).cpu().numpy()
    C_ref = oracle_lib.dequant(acc_ref, sa, sb, zc)
    assert np.array_equal(C.view(np.uint32), C_ref.view(np.uint32))
    # accumulate: C += dequant (the residual store of kernel_vnni_amd64.s:201-234)
    old = np.random.default_rng(1).standard_normal((M, N)).astype(np.float32)
    dC = torch.from_numpy(old.copy()).cuda()
    ops.gemm_u8s8(dA, dB, K=K, sa=dsa, sb=dsb, zc=dzc, C=dC, accumulate=True)
    C2_ref = oracle_lib.dequant(acc_ref, sa, sb, zc, C_old=old)
    assert np.array_equal(dC.cpu().numpy().view(np.uint32), C2_ref.view(np.uint32))


def test_gemm_rows_independent(igdev):
    """A row's output does not depend on the rows computed with it."""
    from indecis_b200 import ops
    A, B, sa, sb, zc = _case(13 * 11, 40, 70, seed=3)
    dA, dB, dsa, dsb, dzc = _dev(A, B, sa, sb, zc)
    all_rows = ops.gemm_u8s8(dA, dB, K=70, sa=dsa, sb=dsb, zc=dzc).cpu().numpy()
    for i in (0, 5, 127, 128, 142):
        one = ops.gemm_u8s8(dA[i:i + 1].contiguous(), dB, K=70, sa=dsa[i:i + 1].contiguous(), sb=dsb,
                            zc=dzc).cpu().numpy()
        assert np.array_equal(one[0].view(np.uint32), all_rows[i].view(np.uint32))


def test_gemm_extreme_operands(igdev, oracle_lib):
    """Maximal magnitudes (255 x -127 over K = 1152): the unsigned-offset sum
    exceeds 2^24, so float(acc) rounds exactly as the reference's VCVTDQ2PS."""
    from indecis_b200 import ops
    M, N, K = 130, 48, 1152
    A = np.full((M, K), 255, np.uint8)
    A[1::2] = 1
    B = np.full((N, K), -127, np.int8)
    B[::3] = 127
    sa = np.full(M, 0.01, np.float32)
    sb = np.full(N, 0.02, np.float32)
    zc = (128.0 * B.astype(np.int64).sum(1)).astype(np.float32)
    acc_ref = oracle_lib.gemm_u8s8(A, B)
    assert np.abs(acc_ref).max() > 2 ** 24
    dA, dB, dsa, dsb, dzc = _dev(A, B, sa, sb, zc)
    assert np.array_equal(ops.gemm_u8s8(dA, dB, int32_out=True).cpu().numpy(), acc_ref)
    C = ops.gemm_u8s8(dA, dB, sa=dsa, sb=dsb, zc=dzc).cpu().numpy()
    assert np.array_equal(C.view(np.uint32), oracle_lib.dequant(acc_ref, sa, sb, zc).view(np.uint32))


@pytest.mark.parametrize("M", [128, 4096])
@pytest.mark.parametrize("N,K", [(768, 256), (256, 384), (2304, 768), (768, 1152)])
def test_gemm_sweep_shapes(igdev, oracle_lib, M, N, K):
    """BASELINE config 2 shapes (M = 65536 is covered by the bench's own checksum)."""
    from indecis_b200 import ops
    A, B, sa, sb, zc = _case(M, N, K, seed=N + K)
    dA, dB, dsa, dsb, dzc = _dev(A, B, sa, sb, zc)
    acc = ops.gemm_u8s8(dA, dB, int32_out=True).cpu().numpy()
    rows = np.r_[0:64, M - 64:M]
    ref = oracle_lib.gemm_u8s8(np.ascontiguousarray(A[rows]), B)
    assert np.array_equal(acc[rows], ref)
    C = ops.gemm_u8s8(dA, dB, sa=dsa, sb=dsb, zc=dzc).cpu().numpy()
    assert np.array_equal(C[rows].view(np.uint32), oracle_lib.dequant(ref, sa[rows], sb, zc).view(np.uint32))
    # size-independent property over all rows: exact integer product vs int64 numpy
    full = (A.astype(np.int64) @ B.astype(np.int64).T)
    assert np.array_equal(acc.astype(np.int64), full)


def _geglu_quant_ref(oracle_lib, A, B, K, I, sa, sb, zc):
    """Wi product, GeGLU (interleaved rows: per 128 columns the GELU inputs,
    then their gates) and quantizeA of each output row, on the oracle."""
    acc = oracle_lib.gemm_u8s8(np.ascontiguousarray(A[:, :K]), np.ascontiguousarray(B[:, :K]))
    z = oracle_lib.dequant(acc, sa, sb, zc)
    j = np.arange(I)
    inp = z[:, 256 * (j // 128) + j % 128]
    gate = z[:, 256 * (j // 128) + 128 + j % 128]
    g = oracle_lib.gelu_mul(inp, gate).reshape(inp.shape)
    return oracle_lib.quantize_a(g)


@pytest.mark.parametrize("M,I,K", [(300, 384, 256), (1, 128, 256), (15360, 384, 256), (777, 1024, 384),
                                   (129, 256, 96)])
def test_gemm_geglu_quant_bitexact(igdev, oracle_lib, M, I, K):
    """The Wi GEMM whose epilogue computes GeGLU and quantizes each output row
    over the cluster of its column tiles equals the oracle's MatMul8N,
    GeluMul and quantizeA (internal/modernbert/infer.go:416-423,
    linalg/int8.go:157-191) bit for bit: bytes and row scales, many row
    blocks per cluster (15360 rows), clusters of 1 to 8 CTAs, and rows that
    take the clamped path: a NaN row scale (NaN values), a huge one (values
    that overflow to infinity), a zero one (a zero row) and a tiny one
    (subnormal outputs and scale)."""
    from indecis_b200 import ops
    A, B, sa, sb, zc = _case(M, 2 * I, K, seed=M + I)
    special = {3: np.nan, 4: 1e30, 5: 0.0, 6: 1e-30}
    for r, v in special.items():
        if r < M:
            sa[r] = v
    q_ref, s_ref = _geglu_quant_ref(oracle_lib, A, B, K, I, sa, sb, zc)
    dA, dB, dsa, dsb, dzc = _dev(A, B, sa, sb, zc)
    ldq = I + 16
    q, s = ops.gemm_geglu_quant(dA, dB, I, dsa, dsb, dzc, K=K, ldq=ldq)
    q, s = q.cpu().numpy(), s.cpu().numpy()
    assert np.array_equal(q[:, :I], q_ref)
    assert (q[:, I:] == 0xAB).all()  # nothing written past the row's I bytes
    assert np.array_equal(s.view(np.uint32), s_ref.view(np.uint32))


def test_gemm_residual_subnormal(igdev, oracle_lib):
    """The residual store x + dequant through the TMA reduce-add keeps IEEE
    addition on subnormal operands (the reference's VADDPS with no flush to
    zero): subnormal old values, subnormal dequantized values, and sums that
    cross the normal boundary."""
    from indecis_b200 import ops
    M, N, K = 260, 256, 256
    A, B, sa, sb, zc = _case(M, N, K, seed=11)
    sa[:] = np.float32(1e-41)  # dequantized values around 1e-41 .. 1e-36, many subnormal
    sa[::7] = np.float32(1e-3)
    acc_ref = oracle_lib.gemm_u8s8(np.ascontiguousarray(A[:, :K]), np.ascontiguousarray(B[:, :K]))
    rng = np.random.default_rng(5)
    tiny = np.float32(1.17549435e-38)
    old = (rng.uniform(-4, 4, (M, N)) * tiny).astype(np.float32)  # subnormal and just-normal values
    old[1::5] = rng.standard_normal((len(range(1, M, 5)), N)).astype(np.float32)
    dA, dB, dsa, dsb, dzc = _dev(A, B, sa, sb, zc)
    dC = torch.from_numpy(old.copy()).cuda()
    ops.gemm_u8s8(dA, dB, K=K, sa=dsa, sb=dsb, zc=dzc, C=dC, accumulate=True)
    want = oracle_lib.dequant(acc_ref, sa, sb, zc, C_old=old)
    got = dC.cpu().numpy()
    assert (np.abs(want[np.abs(want) > 0]) < tiny).any()  # subnormal results are present
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
