"""Config.validate (internal/modernbert/model.go:64-80): every error case, with
the reference's messages, through the host mirror (Config.validate) and
through the C ABI (ig_model_create refuses the config before any device work,
so these run without a GPU)."""
import ctypes as C
import dataclasses

import numpy as np
import pytest


def _cfg(**kw):
    from indecis_b200 import synthetic as S
    from indecis_b200.model import Config
    c = Config.from_dict(S.tiny(layers=2, hidden=128, heads=2, intermediate=192, vocab=100))
    return dataclasses.replace(c, **kw)


CASES = [
    (dict(hidden_size=0), "modernbert: invalid dimensions"),
    (dict(num_hidden_layers=0), "modernbert: invalid dimensions"),
    (dict(num_attention_heads=-1), "modernbert: invalid dimensions"),
    (dict(intermediate_size=0), "modernbert: invalid dimensions"),
    (dict(vocab_size=0), "modernbert: invalid dimensions"),
    (dict(num_attention_heads=3), "modernbert: hidden_size 128 incompatible with 3 heads"),
    (dict(hidden_size=126, num_attention_heads=2), "modernbert: hidden_size 126 incompatible with 2 heads"),
    (dict(global_attn_every_n_layers=0), "modernbert: invalid attention windows"),
    (dict(local_attention=0), "modernbert: invalid attention windows"),
]
HOST_ONLY = [
    (dict(hidden_activation="silu"), 'modernbert: activation "silu" not supported'),
    (dict(attention_bias=True), "modernbert: biases are not supported"),
    (dict(mlp_bias=True), "modernbert: biases are not supported"),
    (dict(norm_bias=True), "modernbert: biases are not supported"),
    (dict(classifier_pooling="max"), 'modernbert: pooling "max" not supported'),
]


@pytest.mark.parametrize("kw,msg", CASES + HOST_ONLY)
def test_validate_host(kw, msg):
    from indecis_b200.model import ModernBertError
    with pytest.raises(ModernBertError) as e:
        _cfg(**kw).validate()
    assert str(e.value) == msg


def test_validate_accepts_the_configs():
    from indecis_b200 import synthetic as S
    from indecis_b200.model import Config
    for d in (S.C1, S.C4):
        Config.from_dict(d).validate()
    _cfg(classifier_pooling="").validate()
    _cfg(classifier_pooling="cls").validate()


def _weights(layers, hidden, inter, vocab):
    z = lambda *s: np.zeros(s, np.float32)
    keep = [z(vocab, hidden), z(hidden), z(hidden)]
    mats = {k: [f() for _ in range(layers)] for k, f in dict(
        attn_norm=lambda: z(hidden), wqkv=lambda: z(3 * hidden, hidden), wo=lambda: z(hidden, hidden),
        mlp_norm=lambda: z(hidden), wi=lambda: z(2 * inter, hidden), wo_mlp=lambda: z(hidden, inter)).items()}
    return keep, mats


@pytest.mark.parametrize("kw,msg", CASES + [(dict(pooling=7), "modernbert: pooling not supported")])
def test_validate_c_abi(kw, msg):
    from indecis_b200 import _capi
    lib = _capi.load()
    pooling = kw.pop("pooling", None)
    c = _cfg(**kw)
    L = max(c.num_hidden_layers, 1)
    keep, mats = _weights(L, max(c.hidden_size, 1), max(c.intermediate_size, 1), max(c.vocab_size, 1))
    arrs = {k: (C.c_void_p * L)(*[a.ctypes.data for a in v]) for k, v in mats.items()}
    w = _capi.IgWeights(tok_embeddings=keep[0].ctypes.data, emb_norm=keep[1].ctypes.data,
                        final_norm=keep[2].ctypes.data,
                        **{k: C.cast(v, C.POINTER(C.c_void_p)) for k, v in arrs.items()})
    cc = c.to_c()
    if pooling is not None:
        cc.pooling = pooling
    h = C.c_void_p()
    rc = lib.ig_model_create(C.byref(cc), C.byref(w), 0, C.byref(h))
    assert rc == _capi.IG_ERR_BAD_ARG
    assert _capi.last_error() == msg
    assert not h.value
