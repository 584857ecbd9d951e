"""Per-operation entry points of libindecis_b200.so on torch CUDA tensors.

Thin wrappers: each checks shapes and dtypes, passes device pointers and the
current torch stream to the C ABI, and raises on a non-zero status. Used by
the parity tests and the GEMM sweep of bench.py.
"""
from __future__ import annotations

import numpy as np
import torch

from . import _capi


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _ptr(t):
    return None if t is None else t.data_ptr()


def _need(t, dtype, name):
    if t.dtype != dtype or not t.is_cuda or not t.is_contiguous():
        raise ValueError(f"{name}: expected a contiguous CUDA {dtype} tensor")


def gemm_u8s8(A, B, K=None, sa=None, sb=None, zc=None, C=None, accumulate=False, int32_out=False):
    """acc = A . B^T (A uint8 [M][lda], B int8 [N][ldb]); returns acc (int32) or
    the dequantized f32 C (written in place when C is given)."""
    _need(A, torch.uint8, "A")
    _need(B, torch.int8, "B")
    M, lda = A.shape
    N, ldb = B.shape
    K = K if K is not None else lda
    L = _capi.load()
    if int32_out:
        acc = torch.empty((M, N), dtype=torch.int32, device=A.device)
        _capi.check(L.ig_gemm_u8s8(_ptr(A), lda, _ptr(B), ldb, M, N, K, None, None, None, None, N, 0, _ptr(acc),
                                   _stream()))
        return acc
    for t, n in ((sa, "sa"), (sb, "sb"), (zc, "zc")):
        _need(t, torch.float32, n)
    if C is None:
        C = torch.empty((M, N), dtype=torch.float32, device=A.device)
        accumulate = False
    _need(C, torch.float32, "C")
    _capi.check(L.ig_gemm_u8s8(_ptr(A), lda, _ptr(B), ldb, M, N, K, _ptr(sa), _ptr(sb), _ptr(zc), _ptr(C),
                               C.shape[1], 1 if accumulate else 0, None, _stream()))
    return C


def gemm_geglu_quant(A, B, I, sa, sb, zc, K=None, ldq=None):
    """The Wi product with the GeGLU epilogue and the output quantized per
    row in the same kernel: B int8 [2I][ldb], rows interleaved per 128 (GELU
    inputs, then gates). Returns (q uint8 [M][ldq], scales [M])."""
    _need(A, torch.uint8, "A")
    _need(B, torch.int8, "B")
    for t, n in ((sa, "sa"), (sb, "sb"), (zc, "zc")):
        _need(t, torch.float32, n)
    M, lda = A.shape
    N, ldb = B.shape
    if N != 2 * I:
        raise ValueError("B must hold 2I rows")
    K = K if K is not None else lda
    ldq = ldq or I
    q = torch.full((M, ldq), 0xAB, dtype=torch.uint8, device=A.device)
    s = torch.full((M,), float("nan"), dtype=torch.float32, device=A.device)
    _capi.check(_capi.load().ig_gemm_geglu_quant(_ptr(A), lda, _ptr(B), ldb, M, I, K, _ptr(sa), _ptr(sb), _ptr(zc),
                                                 _ptr(q), ldq, _ptr(s), _stream()))
    return q, s


def quantize_rows(x, ldq=None):
    _need(x, torch.float32, "x")
    M, K = x.shape
    ldq = ldq or K
    q = torch.empty((M, ldq), dtype=torch.uint8, device=x.device)
    sa = torch.empty(M, dtype=torch.float32, device=x.device)
    _capi.check(_capi.load().ig_quantize_rows(_ptr(x), K, M, K, _ptr(q), ldq, _ptr(sa), _stream()))
    return q, sa


def layernorm_quant(x, gamma, eps=1e-5, simd_lanes=8, want_q=True):
    _need(x, torch.float32, "x")
    _need(gamma, torch.float32, "gamma")
    M, H = x.shape
    xn = torch.empty_like(x)
    q = torch.empty((M, H), dtype=torch.uint8, device=x.device) if want_q else None
    sa = torch.empty(M, dtype=torch.float32, device=x.device) if want_q else None
    _capi.check(_capi.load().ig_layernorm_quant(_ptr(x), _ptr(gamma), M, H, eps, simd_lanes, _ptr(xn), _ptr(q), H,
                                                _ptr(sa), _stream()))
    return xn, q, sa


def pack_b8(w, ldq=None):
    _need(w, torch.float32, "w")
    n, k = w.shape
    ldq = ldq or ((k + 15) // 16 * 16)
    q = torch.empty((n, ldq), dtype=torch.int8, device=w.device)
    s = torch.empty(n, dtype=torch.float32, device=w.device)
    zc = torch.empty(n, dtype=torch.float32, device=w.device)
    cs = torch.empty(n, dtype=torch.int32, device=w.device)
    _capi.check(_capi.load().ig_pack_b8(_ptr(w), n, k, _ptr(q), ldq, _ptr(s), _ptr(zc), _ptr(cs), _stream()))
    return q, s, zc, cs


def attention(qkv, hidden, heads, offs, window, simd_lanes=8):
    _need(qkv, torch.float32, "qkv")
    offs = np.ascontiguousarray(offs, np.int64)
    N = int(offs[-1])
    ctx = torch.full((N, hidden), float("nan"), dtype=torch.float32, device=qkv.device)
    _capi.check(_capi.load().ig_attention(_ptr(qkv), hidden, heads, offs.ctypes.data, len(offs) - 1, window,
                                          simd_lanes, _ptr(ctx), _stream()))
    return ctx


def device_error(reset=True) -> int:
    return _capi.load().ig_device_error(1 if reset else 0)
