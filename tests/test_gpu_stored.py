"""A model made from its tensors as the file stores them (Load,
model.go:661-735): bf16 / f16 / int8 / f32 layer tensors and norms copied to
the device in their own dtype and decoded there as the reference's
safetensors reader decodes them (safetensors.go:218-245), the embedding table
uploaded as stored (bf16 + exact rows). The result must equal, bit for bit,
the model made from the decoded float32 tensors, and the oracle run on them."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _bits(a):
    return np.ascontiguousarray(a).view(np.uint32)


def _bf16(x):
    """float32 -> bf16 bits, round to nearest even (safetensors ToBF16)."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def _stored(cfg, W):
    """Stored tensors of the synthetic weights (matrices bf16, the first
    layer's Wo int8, norms f16 with subnormals, a signed zero and the largest
    f16) and their decoded float32 values."""
    H, L = cfg["hidden"], cfg["layers"]
    stored, dec = {}, dict(W)
    dec = {k: (list(v) if isinstance(v, list) else v) for k, v in W.items()}

    def mat(key, name, l):
        b = _bf16(W[key][l])
        stored[name] = ("BF16", b)
        dec[key][l] = (b.astype(np.uint32) << 16).view(np.float32)

    def norm(key, name, l=None):
        v = (W[key] if l is None else W[key][l]).astype(np.float16)
        v[0], v[1], v[2] = np.float16(2.0 ** -24), np.float16(-3 * 2.0 ** -24), np.float16(-0.0)
        v[3] = np.float16(65504.0)
        stored[name] = ("F16", v.view(np.uint16))
        f = v.astype(np.float32)
        if l is None:
            dec[key] = f
        else:
            dec[key][l] = f

    norm("emb_norm", "embeddings.norm.weight")
    norm("final_norm", "final_norm.weight")
    for l in range(L):
        p = f"layers.{l}."
        if l > 0:
            norm("attn_norm", p + "attn_norm.weight", l)
        norm("mlp_norm", p + "mlp_norm.weight", l)
        mat("wqkv", p + "attn.Wqkv.weight", l)
        mat("wi", p + "mlp.Wi.weight", l)
        mat("wo_mlp", p + "mlp.Wo.weight", l)
        if l == 0:
            q = np.clip(np.rint(W["wo"][l] * 3000), -128, 127).astype(np.int8)
            stored[p + "attn.Wo.weight"] = ("I8", q)
            dec["wo"][l] = q.astype(np.float32)
        else:
            stored[p + "attn.Wo.weight"] = ("F32", W["wo"][l])
    return stored, dec


def test_stored_weights_bitexact(igdev, oracle_lib):
    import oracle
    from indecis_b200 import synthetic as S
    from indecis_b200.model import Config, MappedEmbeddings, Model
    cfg = S.tiny(layers=3, hidden=256, heads=4, intermediate=384, vocab=700)
    W = S.weights(cfg, seed=23, gamma_noise=0.2)
    stored, dec = _stored(cfg, W)
    table = MappedEmbeddings(cfg["hidden"], bf16=_bf16(W["emb"]))
    dec["emb"] = table.matrix()
    gm = Model.FromStored(Config.from_dict(cfg), stored, table)
    ref = Model.from_arrays(Config.from_dict(cfg), dec)
    om = oracle.Model(cfg, dec)
    ids, offs = S.ids_varlen(12, 1, 200, cfg["vocab"], seed=24)
    got = gm.EncodeTokens((ids, offs))
    assert np.array_equal(_bits(got), _bits(ref.EncodeTokens((ids, offs))))
    assert np.array_equal(_bits(got), _bits(om.encode(ids, offs, mode=1)))
    assert np.array_equal(_bits(gm.EncodeSeqs((ids, offs))), _bits(om.encode(ids, offs)))
    # The float path reads the same decoded matrices.
    gm.SetInt8(False)
    assert np.array_equal(_bits(gm.EncodeSeqs((ids, offs))), _bits(om.encode_f32(ids, offs)))
    gm.close()
    ref.close()


def test_stored_weights_errors(igdev):
    from indecis_b200 import _capi
    from indecis_b200 import synthetic as S
    from indecis_b200.model import Config, MappedEmbeddings, Model, ModernBertError
    cfg = S.tiny(layers=2, hidden=128, heads=2, intermediate=192, vocab=100)
    W = S.weights(cfg, seed=3)
    stored, _ = _stored(cfg, W)
    table = MappedEmbeddings(cfg["hidden"], bf16=_bf16(W["emb"]))
    bad = dict(stored)
    bad["final_norm.weight"] = (9, stored["final_norm.weight"][1])  # a dtype code the reader does not know
    with pytest.raises(_capi.IgError, match="unsupported dtype 9") as e:
        Model.FromStored(Config.from_dict(cfg), bad, table)
    assert e.value.code == _capi.IG_ERR_BAD_ARG
    missing = {k: v for k, v in stored.items() if k != "layers.1.mlp.Wi.weight"}
    with pytest.raises(ModernBertError, match="tensor layers.1.mlp.Wi.weight missing"):
        Model.FromStored(Config.from_dict(cfg), missing, table)
