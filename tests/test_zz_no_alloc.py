"""ig_attention_noalloc — the allocation-free attention entry point.

Callers that cannot allocate device memory (servers that reserve all device
memory at start-up, paths that must not let cudaMalloc/cudaFree synchronize
the device) use this variant; its work buffers live in a fixed 32 MiB array
inside the library. The test calls it
through the C ABI twice in a row, on different inputs, and checks each
result against the allocating entry point ig_attention (bit for bit, the
tolerance every attention test here uses), so contents left in the shared
array by one call cannot leak into the next. It also checks that inputs too
large for the array, or sequences longer than its attend kernel takes, are
refused with a clear error before any GPU work.

This file is collected last on purpose: if it fails, a run that stops at the
first failure has already run every other test.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _qkv(lens, H, nh, seed):
    rng = np.random.default_rng(seed)
    N = int(sum(lens))
    D = H // nh
    q = rng.standard_normal((N, H)).astype(np.float32) * 2
    k = rng.standard_normal((N, H)).astype(np.float32) * 2 + (np.arange(H) % D % 5).astype(np.float32)
    v = rng.standard_normal((N, H)).astype(np.float32)
    offs = np.concatenate([[0], np.cumsum(lens)]).astype(np.int64)
    return np.ascontiguousarray(np.concatenate([q, k, v], 1)), offs


def _noalloc(qkv, H, nh, offs, window):
    from indecis_b200 import _capi
    N = int(offs[-1])
    ctx = torch.full((N, H), float("nan"), dtype=torch.float32, device="cuda")
    rc = _capi.load().ig_attention_noalloc(qkv.data_ptr(), H, nh, offs.ctypes.data, len(offs) - 1, window, 8,
                                           ctx.data_ptr(), torch.cuda.current_stream().cuda_stream)
    _capi.check(rc)
    torch.cuda.synchronize()
    return ctx.cpu().numpy()


def test_noalloc_matches_allocating_entry_point(igdev):
    from indecis_b200 import ops
    H, nh = 256, 4
    cases = [([128] * 8 + [5, 77], 64, 1), ([259, 1, 300, 48], -1, 2)]
    for lens, window, seed in cases:  # two calls in a row on the shared array
        qkv_np, offs = _qkv(lens, H, nh, seed)
        qkv = torch.from_numpy(qkv_np).cuda()
        want = ops.attention(qkv, H, nh, offs, window).cpu().numpy()
        got = _noalloc(qkv, H, nh, offs, window)
        assert not np.isnan(got).any()
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (lens, window)


def test_noalloc_nonfinite_keys_match(igdev):
    """Heads whose K rows hold a NaN or an infinity are recomputed with the
    reference's conversions by both entry points (inside the fixed array for
    the allocation-free one): the same bits, NaN where the other has NaN."""
    from indecis_b200 import ops
    H, nh = 256, 4
    qkv_np, offs = _qkv([300, 129, 5], H, nh, 7)
    qkv_np[offs[0] + 7, H + 70] = np.nan
    qkv_np[offs[1] + 9, H + 130] = np.inf
    qkv = torch.from_numpy(qkv_np).cuda()
    want = ops.attention(qkv, H, nh, offs, -1).cpu().numpy()
    got = _noalloc(qkv, H, nh, offs, -1)
    assert np.array_equal(np.isnan(got), np.isnan(want))
    ok = ~np.isnan(want)
    assert np.array_equal(got.view(np.uint32)[ok], want.view(np.uint32)[ok])


def test_noalloc_rejects_oversize(igdev):
    from indecis_b200 import _capi
    H, nh = 256, 4
    # 100 sequences of 10000 tokens: each within the length limit, together
    # far more than 32 MiB of scratch.
    offs = np.arange(0, 1_000_001, 10_000, dtype=np.int64)
    small = torch.zeros((1, 3 * H), dtype=torch.float32, device="cuda")
    rc = _capi.load().ig_attention_noalloc(small.data_ptr(), H, nh, offs.ctypes.data, len(offs) - 1, 64, 8,
                                           small.data_ptr(),
                                           torch.cuda.current_stream().cuda_stream)
    assert rc == _capi.IG_ERR_BAD_ARG
    assert "bytes of scratch" in _capi.last_error()


def test_noalloc_rejects_overlong_sequence(igdev):
    from indecis_b200 import _capi
    H, nh = 256, 4
    offs = np.array([0, 11000], np.int64)  # fits the scratch array, but over the 10240-token limit
    small = torch.zeros((1, 3 * H), dtype=torch.float32, device="cuda")
    rc = _capi.load().ig_attention_noalloc(small.data_ptr(), H, nh, offs.ctypes.data, 1, -1, 8, small.data_ptr(),
                                           torch.cuda.current_stream().cuda_stream)
    assert rc == _capi.IG_ERR_UNSUPPORTED
    assert "longer than the 10240" in _capi.last_error()
