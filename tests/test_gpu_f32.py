"""The encoder's float32 path on the device (SetInt8(false)), bit for bit
against the oracle's restatement (or_encode_f32): ragged batches whose
sequences span several key blocks of attendBlocks, global and local layers,
token states and pooled outputs, C4's layer shape, and the switch back to
int8."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _bits(a):
    return np.ascontiguousarray(a).view(np.uint32)


def _models(cfg, seed):
    import oracle
    from indecis_b200 import synthetic as S
    from indecis_b200.model import Config, Model
    W = S.weights(cfg, seed=seed, gamma_noise=0.1)
    gm = Model.from_arrays(Config.from_dict(cfg), W)
    gm.SetInt8(False)
    return oracle.Model(cfg, W), gm


@pytest.mark.parametrize("lo,hi", [(1, 64), (1, 330), (120, 520)])
def test_f32_ragged_bitexact(igdev, oracle_lib, lo, hi):
    from indecis_b200 import synthetic as S
    cfg = S.tiny(layers=3, hidden=128, heads=2, intermediate=192, vocab=700)
    om, gm = _models(cfg, seed=3)
    ids, offs = S.ids_varlen(9, lo, hi, cfg["vocab"], seed=lo + hi, lo=0)
    assert np.array_equal(_bits(gm.EncodeTokens((ids, offs))), _bits(om.encode_f32(ids, offs, mode=1, threads=8)))
    assert np.array_equal(_bits(gm.EncodeSeqs((ids, offs))), _bits(om.encode_f32(ids, offs, threads=8)))


def test_f32_c1_and_c4_shapes(igdev, oracle_lib):
    from indecis_b200 import synthetic as S
    om, gm = _models(S.C1, seed=42)
    ids, offs = S.ids_fixed(6, 128, S.C1["vocab"], seed=1)
    assert np.array_equal(_bits(gm.EncodeSeqs((ids, offs))), _bits(om.encode_f32(ids, offs, threads=8)))
    cfg = dict(S.C4)
    cfg.update(layers=2, vocab=3000)
    om, gm = _models(cfg, seed=7)
    ids, offs = S.ids_varlen(4, 30, 300, cfg["vocab"], seed=4)
    assert np.array_equal(_bits(gm.EncodeTokens((ids, offs))), _bits(om.encode_f32(ids, offs, mode=1, threads=8)))


def test_switch_back_to_int8(igdev, oracle_lib):
    from indecis_b200 import synthetic as S
    cfg = S.tiny(layers=2, hidden=128, heads=2, intermediate=192, vocab=500)
    om, gm = _models(cfg, seed=5)
    ids, offs = S.ids_varlen(5, 1, 100, cfg["vocab"], seed=6)
    f = gm.EncodeSeqs((ids, offs))
    gm.SetInt8(True)
    q = gm.EncodeSeqs((ids, offs))
    assert np.array_equal(_bits(q), _bits(om.encode(ids, offs)))
    assert np.array_equal(_bits(f), _bits(om.encode_f32(ids, offs)))
