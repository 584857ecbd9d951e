"""The SigLIP vision tower on the device (ig_vision_*), bit for bit against
the oracle (oracle/siglip.cpp): every layer's intermediates through the dump
path, the patch features of Forward at a layer and at the end, the pooled
embeddings of Embed; the C5 layer shape (hidden 768, 12 heads, MLP 3072,
196 patches); more than 32 outlier channels; batch independence; errors.
Mirrors internal/siglip/siglip_test.go (TestForwardLayers) on synthetic
weights."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _bits(a):
    return np.ascontiguousarray(a).view(np.uint32)


def _models(cfg, seed=1, **kw):
    import oracle
    from indecis_b200 import synthetic as S
    from indecis_b200.siglip import Vision, VisionConfig
    W = S.siglip_weights(cfg, seed=seed, **kw)
    return oracle.SigLIP(cfg, W), Vision.from_arrays(VisionConfig.from_dict(cfg), W)


def _check_dump(dg, do, layers_checked=None):
    for k in ("h1q", "h2q", "mq"):
        assert np.array_equal(dg[k], do[k]), k
    for k in ("x_embed", "h1q_s", "qkv", "attn", "x_attn", "h2q_s", "mlp", "mq_s", "x_mlp"):
        assert np.array_equal(_bits(dg[k]), _bits(do[k])), k
    assert np.array_equal(dg["noutliers"], do["noutliers"])
    for i, c in enumerate(do["noutliers"]):
        assert np.array_equal(dg["outliers"][i, :c], do["outliers"][i, :c])


@pytest.mark.parametrize("cfg_kw", [dict(), dict(image_size=48, patch_size=8, layers=3), dict(image_size=60,
                                                                                             patch_size=6)])
def test_tiny_tower_bitexact(igdev, oracle_lib, cfg_kw):
    from indecis_b200 import synthetic as S
    cfg = S.siglip_tiny(**cfg_kw)
    om, gm = _models(cfg)
    px = S.pixels(5, cfg["image_size"], seed=4)
    for layer in range(cfg["layers"]):
        pa, po, do = om.forward(px, dump_layer=layer)
        dg, pg = gm.dump(px, layer)
        _check_dump(dg, do)
        assert np.array_equal(_bits(pg), _bits(po))
    gp, ge = gm.Forward(px, layer=0, pool=True)
    assert np.array_equal(_bits(gp), _bits(pa)) and np.array_equal(_bits(ge), _bits(po))
    assert np.array_equal(_bits(gm.Embed(px)), _bits(po))


def test_forward_layers(igdev, oracle_lib):
    """TestForwardLayers (siglip_test.go:258): a layer's patch features with
    and without pooling, and the pooled vector beside them."""
    from indecis_b200 import synthetic as S
    cfg = S.siglip_tiny(layers=3)
    om, gm = _models(cfg, seed=3)
    px = S.pixels(3, cfg["image_size"], seed=8)
    for layer in (1, 2, 3):
        want, _ = om.forward(px, layer=layer, pooled=False)
        got, none = gm.Forward(px, layer=layer, pool=False)
        assert none is None and np.array_equal(_bits(got), _bits(want))
        got2, emb = gm.Forward(px, layer=layer, pool=True)
        assert np.array_equal(_bits(got2), _bits(want))
        assert np.array_equal(_bits(emb), _bits(om.forward(px, pooled=True, patches=False)[1]))


def test_many_outliers(igdev, oracle_lib):
    """More than 32 channels above the threshold: the reference keeps the 32
    largest in its selection-sort order (linalg/int8.go:313-324)."""
    from indecis_b200 import synthetic as S
    cfg = S.siglip_tiny(mlp=512)
    om, gm = _models(cfg, seed=6, massive=48, massive_gain=8.0)
    px = S.pixels(3, cfg["image_size"], seed=2)
    T, M = 16, cfg["mlp"]
    _, po, do = om.forward(px, dump_layer=0)
    colmax = np.abs(do["mlp"]).reshape(3, T, M).max(1)
    mean = colmax.astype(np.float32).cumsum(1, dtype=np.float32)[:, -1] / np.float32(M)
    assert ((colmax > (6 * mean)[:, None]).sum(1) > 32).all()  # the selection path runs
    assert (do["noutliers"] == 32).all()
    for layer in (0, 1):
        _, po, do = om.forward(px, dump_layer=layer)
        dg, pg = gm.dump(px, layer)
        _check_dump(dg, do)
        assert np.array_equal(_bits(pg), _bits(po))


def test_c5_layer_shape(igdev, oracle_lib):
    """C5's layer shape (hidden 768, 12 heads, MLP 3072, 224 px / 16: 196
    patches) with two layers: the ragged softmax tail (196 = 24 x 8 + 4),
    K = 768 and 3072 products, three 256-deep blocks in the float32 products."""
    from indecis_b200 import synthetic as S
    cfg = dict(S.C5)
    cfg.update(layers=2)
    om, gm = _models(cfg, seed=9)
    px = S.pixels(2, cfg["image_size"], seed=10)
    pa, po, do = om.forward(px, dump_layer=1, threads=2)
    dg, pg = gm.dump(px, 1)
    _check_dump(dg, do)
    assert np.array_equal(_bits(pg), _bits(po))
    gp, ge = gm.Forward(px, pool=True)
    assert np.array_equal(_bits(gp), _bits(pa)) and np.array_equal(_bits(ge), _bits(po))


def test_batch_independence(igdev, oracle_lib):
    from indecis_b200 import synthetic as S
    cfg = S.siglip_tiny()
    _, gm = _models(cfg, seed=12)
    px = S.pixels(7, cfg["image_size"], seed=13)
    whole = gm.Embed(px)
    for i in (0, 3, 6):
        assert np.array_equal(_bits(gm.Embed(px[i])), _bits(whole[i:i + 1]))


def test_errors(igdev):
    from indecis_b200 import synthetic as S
    from indecis_b200.siglip import SiglipError, Vision, VisionConfig
    cfg = S.siglip_tiny()
    gm = Vision.from_arrays(VisionConfig.from_dict(cfg), S.siglip_weights(cfg))
    px = S.pixels(1, cfg["image_size"])
    with pytest.raises(SiglipError, match="layer 3, the tower has 2"):
        gm.Forward(px, layer=3)
    with pytest.raises(SiglipError, match="pixel values"):
        gm.Embed(np.zeros((3, 8, 8), np.float32))
    bad = dict(cfg)
    bad.update(image_size=30)
    with pytest.raises(SiglipError, match="inconsistent dimensions"):
        Vision.from_arrays(VisionConfig.from_dict(bad), S.siglip_weights(cfg))
