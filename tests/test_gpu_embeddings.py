"""Embedding tables in their stored formats (embeddings.go:9-68,
internal/modernbert/infer.go:12-60): bf16 rows widened exactly (bits << 16)
with float32 rows for the ids listed as exact, and int8 rows times a row
scale. The device gathers and widens them itself; the oracle gets the same
table materialized in float32 (MappedEmbeddings.Row, the reference's Row),
and the encoder outputs must agree bit for bit. The three widths exercise the
three gather kernels (V = 8 register chains, grouped rows, one row per warp)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _bits(a):
    return np.ascontiguousarray(a).view(np.uint32)


def _tables(W, cfg, seed):
    from indecis_b200.model import MappedEmbeddings
    rng = np.random.default_rng(seed)
    V, H = cfg["vocab"], cfg["hidden"]
    emb = W["emb"]
    bf16 = (emb.view(np.uint32) >> 16).astype(np.uint16)  # truncated to bf16
    bf16[::7] ^= 1  # and some odd low bits
    exact_ids = rng.choice(V, size=V // 10, replace=False).astype(np.int32)
    exact_ids = np.concatenate([exact_ids, exact_ids[:3]])  # a repeated id: the later row wins
    exact_rows = (rng.standard_normal((len(exact_ids), H)) * 0.05).astype(np.float32)
    mapped = MappedEmbeddings(H, bf16=bf16, exact_ids=exact_ids, exact_rows=exact_rows)
    i8 = rng.integers(-128, 128, size=(V, H), dtype=np.int64).astype(np.int8)
    scale = (rng.uniform(1e-4, 1e-3, V)).astype(np.float32)
    scale[5] = 0.0
    int8 = MappedEmbeddings(H, i8=i8, scale=scale)
    return mapped, int8


@pytest.mark.parametrize("hidden,lanes", [(256, 8), (384, 8), (128, 6)])
def test_embedding_formats_bitexact(igdev, oracle_lib, hidden, lanes):
    import oracle
    from indecis_b200 import synthetic as S
    from indecis_b200.model import Config, Model
    cfg = S.tiny(layers=2, hidden=hidden, heads=hidden // 64, intermediate=384, vocab=600)
    cfg["V"] = lanes
    W = S.weights(cfg, seed=11)
    gm = Model.from_arrays(Config.from_dict(cfg), W)
    ids, offs = S.ids_varlen(9, 1, 150, cfg["vocab"], seed=12, lo=0)
    for table in _tables(W, cfg, seed=hidden):
        gm.SetEmbeddingTable(table)
        Wm = dict(W)
        Wm["emb"] = table.matrix()
        om = oracle.Model(cfg, Wm)
        assert np.array_equal(_bits(gm.EncodeTokens((ids, offs))), _bits(om.encode(ids, offs, mode=1)))
        assert np.array_equal(_bits(gm.EncodeSeqs((ids, offs))), _bits(om.encode(ids, offs)))


def test_embedding_table_errors(igdev):
    import ctypes as C
    from indecis_b200 import _capi
    from indecis_b200 import synthetic as S
    from indecis_b200.model import Config, MappedEmbeddings, Model, ModernBertError
    cfg = S.tiny(layers=1, hidden=128, heads=2, intermediate=192, vocab=100)
    gm = Model.from_arrays(Config.from_dict(cfg), S.weights(cfg))
    bf16 = np.zeros((100, 128), np.uint16)
    with pytest.raises(ModernBertError, match="exact row 100 out of vocabulary"):
        MappedEmbeddings(128, bf16=bf16, exact_ids=[3, 100], exact_rows=np.zeros((2, 128), np.float32))
    with pytest.raises(ModernBertError, match="int8 table"):
        MappedEmbeddings(128, i8=np.zeros(100 * 128 - 1, np.int8), scale=np.ones(100, np.float32))
    # The C ABI checks the ids itself.
    ids = np.array([7, 100], np.int32)
    rows = np.zeros((2, 128), np.float32)
    tab = _capi.IgEmbeddingTable(format=_capi.IG_EMB_BF16, bf16=bf16.ctypes.data, n_exact=2,
                                 exact_ids=ids.ctypes.data, exact_rows=rows.ctypes.data)
    assert _capi.load().ig_model_set_embeddings(gm._h, C.byref(tab)) == _capi.IG_ERR_BAD_ARG
    assert "exact row 100 out of vocabulary" in _capi.last_error()
    bad = _capi.IgEmbeddingTable(format=7)
    assert _capi.load().ig_model_set_embeddings(gm._h, C.byref(bad)) == _capi.IG_ERR_BAD_ARG
