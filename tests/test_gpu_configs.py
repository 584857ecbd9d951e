"""The encoder at the other BASELINE shapes, bit-exact against the oracle.

At full size (the oracle's threaded VNNI path takes seconds to a minute):

  C3 long: 8 sequences of 4096 tokens through the whole C1 model (global
     layers 0 and 3 over all 4096 keys, local layers with the half-window 64);
  C3 varlen: the 256 unpadded sequences of U[8, 512] tokens (seed 3);
  C4: the base model itself (22 layers, vocab 262144, hidden 768, 12 heads,
     intermediate 1152) on four 512-token sequences, pooled and token states.

At reduced sizes:

  C3 (C1's model): two 1024-token sequences (global layers over 1024 keys:
     the attention path for long key ranges) and a ragged batch with lengths
     in [8, 512];
  C4's layer shape (hidden 768, 12 heads of 64, intermediate 1152) with two
     layers (one global, one local) and a smaller vocabulary: the row kernels
     for wide rows, K = 768 / 1152 GEMMs, N = 2304 QKV.

Mirrors internal/modernbert/infer_test.go (EncodeSeqs / EncodeTokens)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _models(cfg, seed=42, gamma_noise=0.1):
    import oracle
    from indecis_b200 import synthetic as S
    from indecis_b200.model import Config, Model
    W = S.weights(cfg, seed=seed, gamma_noise=gamma_noise)
    return oracle.Model(cfg, W), Model.from_arrays(Config.from_dict(cfg), W)


def _bits(a):
    return np.ascontiguousarray(a).view(np.uint32)


def _concat(*batches):
    ids = np.concatenate([b[0] for b in batches]).astype(np.int32)
    offs = [0]
    for b in batches:
        offs.extend((offs[-1] + np.cumsum(np.diff(b[1]))).tolist())
    return ids, np.asarray(offs, np.int64)


def test_c3_long_and_ragged(igdev, oracle_lib):
    from indecis_b200 import synthetic as S
    om, gm = _models(S.C1)
    ids, offs = _concat(S.ids_fixed(2, 1024, S.C1["vocab"], seed=31),
                        S.ids_varlen(24, 8, 512, S.C1["vocab"], seed=3))
    assert np.array_equal(_bits(gm.EncodeSeqs((ids, offs))), _bits(om.encode(ids, offs, threads=8)))
    assert np.array_equal(_bits(gm.EncodeTokens((ids, offs))), _bits(om.encode(ids, offs, mode=1, threads=8)))


def test_c4_layer_shape(igdev, oracle_lib):
    from indecis_b200 import synthetic as S
    cfg = dict(S.C4)
    cfg.update(layers=2, vocab=4096)
    om, gm = _models(cfg, seed=7)
    ids, offs = _concat(S.ids_fixed(6, 96, cfg["vocab"], seed=41),
                        S.ids_varlen(10, 1, 150, cfg["vocab"], seed=42))
    assert np.array_equal(_bits(gm.EncodeSeqs((ids, offs))), _bits(om.encode(ids, offs, threads=8)))
    assert np.array_equal(_bits(gm.EncodeTokens((ids, offs))), _bits(om.encode(ids, offs, mode=1, threads=8)))
    # Every layer's intermediates through the dump path as well.
    ro, do = om.encode(ids, offs, dump_layer=1, threads=8)
    rg, dg = gm.encode_dump((ids, offs), 1)
    for k in ("xq", "cq", "hq", "gq"):
        assert np.array_equal(dg[k], do[k]), k
    for k in ("qkv", "ctx", "x_attn", "x_mlp"):
        assert np.array_equal(_bits(dg[k]), _bits(do[k])), k
    assert np.array_equal(_bits(rg), _bits(ro))


def _host_threads():
    import os
    return max(1, os.cpu_count() or 1)


def test_c3_full_long(igdev, oracle_lib):
    from indecis_b200 import synthetic as S
    om, gm = _models(S.C1)
    ids, offs = S.ids_fixed(8, 4096, S.C1["vocab"], seed=31)
    t = _host_threads()
    assert np.array_equal(_bits(gm.EncodeSeqs((ids, offs))), _bits(om.encode(ids, offs, threads=t, fast=True)))
    assert np.array_equal(_bits(gm.EncodeTokens((ids, offs))),
                          _bits(om.encode(ids, offs, mode=1, threads=t, fast=True)))


def test_c3_long_ragged(igdev, oracle_lib):
    """Sequences of 2048 tokens or more whose lengths are not multiples of the
    128-row statistics stages or of the 64-row quantization tiles (the
    statistics split by RoPE pair, a partial last stage and tile), beside a
    short one, through the whole C1 model with RoPE."""
    from indecis_b200 import synthetic as S
    om, gm = _models(S.C1)
    rng = np.random.default_rng(5)
    lens = [2049, 3001, 7, 2300]
    offs = np.concatenate([[0], np.cumsum(lens)]).astype(np.int64)
    ids = rng.integers(0, S.C1["vocab"], size=int(offs[-1])).astype(np.int32)
    t = _host_threads()
    assert np.array_equal(_bits(gm.EncodeSeqs((ids, offs))), _bits(om.encode(ids, offs, threads=t, fast=True)))
    assert np.array_equal(_bits(gm.EncodeTokens((ids, offs))),
                          _bits(om.encode(ids, offs, mode=1, threads=t, fast=True)))


def test_c3_full_varlen(igdev, oracle_lib):
    from indecis_b200 import synthetic as S
    om, gm = _models(S.C1)
    ids, offs = S.ids_varlen(256, 8, 512, S.C1["vocab"], seed=3)
    t = _host_threads()
    assert np.array_equal(_bits(gm.EncodeSeqs((ids, offs))), _bits(om.encode(ids, offs, threads=t, fast=True)))
    assert np.array_equal(_bits(gm.EncodeTokens((ids, offs))),
                          _bits(om.encode(ids, offs, mode=1, threads=t, fast=True)))


def test_c4_full_model(igdev, oracle_lib):
    from indecis_b200 import synthetic as S
    om, gm = _models(S.C4, seed=42, gamma_noise=0.0)
    ids, offs = S.ids_fixed(4, 512, S.C4["vocab"], seed=41)
    t = _host_threads()
    assert np.array_equal(_bits(gm.EncodeSeqs((ids, offs))), _bits(om.encode(ids, offs, threads=t, fast=True)))
    assert np.array_equal(_bits(gm.EncodeTokens((ids, offs))),
                          _bits(om.encode(ids, offs, mode=1, threads=t, fast=True)))
    gm.close()
