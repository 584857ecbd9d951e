"""int8 attention vs the oracle, bit-exact, over unpadded varlen batches,
local and global (linalg/attention8_test.go:50 TestAttend8 shapes and
windows, :87 TestAttn8Ranges), with NaN-prefilled outputs that must be
fully written."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _qkv(lens, H, nh, seed):
    rng = np.random.default_rng(seed)
    N = int(sum(lens))
    D = H // nh
    q = rng.standard_normal((N, H)).astype(np.float32) * 2
    k = rng.standard_normal((N, H)).astype(np.float32) * 2 + (np.arange(H) % D % 7).astype(np.float32)
    v = rng.standard_normal((N, H)).astype(np.float32)
    return np.ascontiguousarray(np.concatenate([q, k, v], 1)), np.concatenate([[0], np.cumsum(lens)]).astype(np.int64)


def _ref(oracle_lib, qkv, offs, H, nh, window):
    D = H // nh
    out = np.zeros((qkv.shape[0], H), np.float32)
    for s in range(len(offs) - 1):
        a, b = offs[s], offs[s + 1]
        for h in range(nh):
            o = oracle_lib.attn8(qkv[a:b, h * D:(h + 1) * D], qkv[a:b, H + h * D:H + (h + 1) * D],
                                 qkv[a:b, 2 * H + h * D:2 * H + (h + 1) * D], window, np.float32(1 / np.sqrt(D)))
            out[a:b, h * D:(h + 1) * D] = o
    return out


@pytest.mark.parametrize("window", [-1, 8, 64])
@pytest.mark.parametrize("lens", [[1], [5], [17], [48], [100], [128], [259], [1, 5, 17, 48, 100, 259],
                                  [128] * 8, [512, 3, 300]])
def test_attention_bitexact(igdev, oracle_lib, lens, window):
    from indecis_b200 import ops
    H, nh = 256, 4
    qkv, offs = _qkv(lens, H, nh, seed=sum(lens) + window)
    ref = _ref(oracle_lib, qkv, offs, H, nh, window)
    ctx = ops.attention(torch.from_numpy(qkv).cuda(), H, nh, offs, window).cpu().numpy()
    assert not np.isnan(ctx).any()
    assert np.array_equal(ctx.view(np.uint32), ref.view(np.uint32))


def test_attention_long_global(igdev, oracle_lib):
    """A 4096-token global layer (BASELINE config 3 length)."""
    from indecis_b200 import ops
    H, nh = 128, 2
    qkv, offs = _qkv([4096], H, nh, seed=11)
    ref = _ref(oracle_lib, qkv, offs, H, nh, -1)
    ctx = ops.attention(torch.from_numpy(qkv).cuda(), H, nh, offs, -1).cpu().numpy()
    assert np.array_equal(ctx.view(np.uint32), ref.view(np.uint32))


def test_attention_long_ragged(igdev, oracle_lib):
    """Global layers over sequences of 2048 tokens or more with ragged
    lengths (partial statistics stages and quantization tiles, a sequence end
    inside a key tile), beside a short sequence."""
    from indecis_b200 import ops
    H, nh = 128, 2
    lens = [2049, 3, 2222]
    qkv, offs = _qkv(lens, H, nh, seed=29)
    ref = _ref(oracle_lib, qkv, offs, H, nh, -1)
    ctx = ops.attention(torch.from_numpy(qkv).cuda(), H, nh, offs, -1).cpu().numpy()
    assert not np.isnan(ctx).any()
    bad = np.argwhere(ctx.view(np.uint32) != ref.view(np.uint32))
    assert len(bad) == 0, f"{len(np.unique(bad[:, 0]))} rows differ, first {bad[:3].tolist()}"


def _special(qkv, offs, H, cases):
    """Plants the named special values: Q, K, V rows of the first sequence
    and small rows of the second."""
    a, b = int(offs[0]), int(offs[1])
    plant = {
        "q_nan": lambda: qkv.__setitem__((a + 3, 5), np.nan),
        "v_inf": lambda: qkv.__setitem__((a + 11, 2 * H + 200), -np.inf),
        "v_nan": lambda: qkv.__setitem__((a + 13, 2 * H + 10), np.nan),
        "zero_rows": lambda: (qkv.__setitem__((a + 15, slice(0, H)), 0.0),
                              qkv.__setitem__((a + 16, slice(H, 2 * H)), 0.0),
                              qkv.__setitem__((a + 17, slice(2 * H, 3 * H)), 0.0)),
        "tiny_scales": lambda: (qkv.__setitem__((b + 2, slice(0, H)), qkv[b + 2, 0:H] * 1e-40),
                                qkv.__setitem__((b + 4, slice(H, 2 * H)), qkv[b + 4, H:2 * H] * 1e-40)),
        "k_nan": lambda: qkv.__setitem__((a + 7, H + 70), np.nan),
        "k_inf": lambda: qkv.__setitem__((a + 9, H + 130), np.inf),
        "q_inf": lambda: qkv.__setitem__((a + 5, 200), -np.inf),
    }
    for c in cases:
        plant[c]()


def _compare_special(oracle_lib, lens, cases):
    from indecis_b200 import ops
    H, nh = 256, 4
    qkv, offs = _qkv(lens, H, nh, seed=sum(lens) + 5)
    _special(qkv, offs, H, cases)
    ref = _ref(oracle_lib, qkv, offs, H, nh, -1)
    ctx = ops.attention(torch.from_numpy(qkv).cuda(), H, nh, offs, -1).cpu().numpy()
    assert np.array_equal(np.isnan(ctx), np.isnan(ref))
    ok = ~np.isnan(ref)
    bad = np.argwhere(ctx.view(np.uint32)[ok] != ref.view(np.uint32)[ok])
    assert len(bad) == 0, f"{len(bad)} values differ"


@pytest.mark.parametrize("lens", [[96, 128, 17], [300, 129, 5]])
def test_attention_special_values(igdev, oracle_lib, lens):
    """Rows that take the rare quantization branches (sequences up to 128
    tokens and longer ones): a Q row holding a NaN, a NaN and an infinity in V
    columns, all-zero Q, K and V rows, and Q and K rows so small that their
    scale max/127 is subnormal; every output bit as the oracle's (NaN where it
    has NaN)."""
    _compare_special(oracle_lib, lens, ["q_nan", "v_inf", "v_nan", "zero_rows", "tiny_scales"])


@pytest.mark.parametrize("lens", [[96, 128, 17], [300, 129, 5]])
@pytest.mark.parametrize("case", ["k_nan", "k_inf", "q_inf"])
def test_attention_nonfinite_keys(igdev, oracle_lib, case, lens):
    """A NaN or an infinity in a K row makes that head's K column mean
    non-finite: every key of the (sequence, head) then converts with INT_MIN
    in its byte sum (a 128*sum correction far beyond what the tensor-core
    kernels' integer-to-float shortcut covers), and an infinite key makes the
    scores NaN, which the reference carries through ExpShift's clamps into P
    (as INT_MIN in the row's P sum, the row scale 1/qsum unguarded).
    ig_attention recomputes such heads with the reference's conversions: every
    output bit as the oracle's (NaN where it has NaN), short and long
    sequences, a NaN and an infinity in a Q row too."""
    _compare_special(oracle_lib, lens, [case])


def test_attention_accuracy_vs_float(igdev):
    """TestAttend8 bounds: relative error <= 0.03, worst <= 0.25 vs float64."""
    from indecis_b200 import ops
    H, nh = 64, 1
    for n in (5, 48, 259):
        for window in (-1, 8, 64):
            qkv, offs = _qkv([n], H, nh, seed=n * 3 + window)
            ctx = ops.attention(torch.from_numpy(qkv).cuda(), H, nh, offs, window).cpu().numpy().astype(np.float64)
            q, k, v = (qkv[:, i * H:(i + 1) * H].astype(np.float64) for i in range(3))
            s = q @ k.T / np.sqrt(H)
            idx = np.arange(n)
            if window >= 0:
                s[np.abs(idx[:, None] - idx[None, :]) > window] = -np.inf
            p = np.exp(s - s.max(1, keepdims=True))
            want = (p / p.sum(1, keepdims=True)) @ v
            d = ctx - want
            rel = np.sqrt((d ** 2).sum() / (want ** 2).sum())
            assert rel <= 0.03 and np.abs(d).max() <= 0.25, (n, window, rel)


@pytest.mark.parametrize("window", [-1, 64])
def test_attention_many_rows(igdev, oracle_lib, window):
    """Rare rounding differences (one row in thousands) only show over many
    rows: 96 sequences of 1..256 tokens, 4 heads, every row bit-exact."""
    from indecis_b200 import ops
    rng = np.random.default_rng(77 + window)
    lens = rng.integers(1, 257, size=96).tolist()
    H, nh = 256, 4
    qkv, offs = _qkv(lens, H, nh, seed=123 + window)
    ref = _ref(oracle_lib, qkv, offs, H, nh, window)
    ctx = ops.attention(torch.from_numpy(qkv).cuda(), H, nh, offs, window).cpu().numpy()
    bad = np.argwhere(ctx.view(np.uint32) != ref.view(np.uint32))
    assert len(bad) == 0, f"{len(np.unique(bad[:, 0]))} rows differ, first {bad[:3].tolist()}"


@pytest.mark.parametrize("lens", [[257], [384], [385, 511, 640], [1000, 2, 300, 700]])
def test_attention_long_key_tiles(igdev, oracle_lib, lens):
    """Global layers over more than two 128-key tiles: the two-pass kernel
    (row maximum over every tile, then P and O per tile), with sequence ends
    on and off tile boundaries and the ExpShift tail across them; every row of
    every sequence bit-exact."""
    from indecis_b200 import ops
    H, nh = 256, 4
    qkv, offs = _qkv(lens, H, nh, seed=sum(lens) * 7 + 1)
    ref = _ref(oracle_lib, qkv, offs, H, nh, -1)
    ctx = ops.attention(torch.from_numpy(qkv).cuda(), H, nh, offs, -1).cpu().numpy()
    assert not np.isnan(ctx).any()
    bad = np.argwhere(ctx.view(np.uint32) != ref.view(np.uint32))
    assert len(bad) == 0, f"{len(np.unique(bad[:, 0]))} rows differ, first {bad[:3].tolist()}"
