"""Whole int8 encoder on the GPU vs the oracle: every layer's int8
activations, scales and float states bit-exact; pooled outputs, token states
and head logits bit-exact (the spec bound is 1e-4 absolute on logits).
Mirrors internal/modernbert/infer_test.go (EncodeSeqs / EncodeTokens) and
concurrency_test.go:12 (batch composition and concurrency do not change a
sequence's result)."""
import threading

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _models(cfg, seed=42, gamma_noise=0.1):
    import oracle
    from indecis_b200 import synthetic as S
    from indecis_b200.model import Config, Model
    W = S.weights(cfg, seed=seed, gamma_noise=gamma_noise)
    return oracle.Model(cfg, W), Model.from_arrays(Config.from_dict(cfg), W), W


def _bits(a):
    return np.ascontiguousarray(a).view(np.uint32)


@pytest.fixture(scope="module")
def tiny(igdev, oracle_lib):
    from indecis_b200 import synthetic as S
    cfg = S.tiny(layers=4, hidden=256, heads=4, intermediate=384, vocab=1000)
    return (cfg,) + _models(cfg)


def test_layers_bitexact(tiny):
    from indecis_b200 import synthetic as S
    cfg, om, gm, _ = tiny
    ids, offs = S.ids_varlen(7, 1, 300, cfg["vocab"], seed=5)
    for layer in range(cfg["layers"]):
        ro, do = om.encode(ids, offs, dump_layer=layer)
        rg, dg = gm.encode_dump((ids, offs), layer)
        if layer == 0:
            assert np.array_equal(_bits(dg["emb_ln"]), _bits(do["emb_ln"]))
        for k in ("xq", "cq", "hq", "gq"):
            assert np.array_equal(dg[k], do[k]), (layer, k)
        for k in ("xq_s", "cq_s", "hq_s", "gq_s", "qkv", "ctx", "x_attn", "x_mlp"):
            assert np.array_equal(_bits(dg[k]), _bits(do[k])), (layer, k)
        assert np.array_equal(_bits(rg), _bits(ro))


def test_encode_seqs_and_tokens(tiny):
    from indecis_b200 import synthetic as S
    cfg, om, gm, _ = tiny
    ids, offs = S.ids_varlen(9, 1, 200, cfg["vocab"], seed=6)
    seqs = [ids[offs[i]:offs[i + 1]] for i in range(len(offs) - 1)]
    assert np.array_equal(_bits(gm.EncodeSeqs(seqs)), _bits(om.encode(ids, offs, mode=0)))
    assert np.array_equal(_bits(gm.EncodeTokens(seqs)), _bits(om.encode(ids, offs, mode=1)))


def test_c1_batch_bitexact(igdev, oracle_lib):
    """32 x 128 tokens, 6 layers, hidden 256."""
    from indecis_b200 import synthetic as S
    om, gm, _ = _models(S.C1, gamma_noise=0.0)
    ids, offs = S.ids_fixed(32, 128, S.C1["vocab"], seed=1)
    ref = om.encode(ids, offs, threads=8)
    got = gm.EncodeSeqs((ids, offs))
    assert np.array_equal(_bits(got), _bits(ref))


def test_c1_varlen_bitexact(igdev, oracle_lib):
    """C1's dimensions on ragged sequences (1..200 tokens: partial GEMM row
    blocks, the fused short-sequence attention and the tensor-core attention
    for sequences over 128 tokens), through the pooled, per-token and dump
    entry points, bit for bit."""
    from indecis_b200 import synthetic as S
    om, gm, _ = _models(S.C1, gamma_noise=0.1)
    ids, offs = S.ids_varlen(40, 1, 200, S.C1["vocab"], seed=21)
    ref_tok = om.encode(ids, offs, mode=1, threads=8)
    got_tok = gm.EncodeTokens((ids, offs))
    assert np.array_equal(_bits(got_tok), _bits(ref_tok))
    ref = om.encode(ids, offs, threads=8)
    assert np.array_equal(_bits(gm.EncodeSeqs((ids, offs))), _bits(ref))
    out, _ = gm.encode_dump((ids, offs), layer=3)
    assert np.array_equal(_bits(out), _bits(ref))


@pytest.mark.parametrize("hidden,heads", [(256, 4), (128, 2)])
def test_short_sequences_fused_projection(igdev, oracle_lib, hidden, heads):
    """Batches whose sequences all fit 128 tokens take the attention kernel
    that computes the QKV projection itself (one and two 128-byte K blocks):
    ragged lengths 1..128
    (the last sequence's 128-row operand box runs past the batch), an empty
    sequence between them, and an all-128 batch, bit for bit through the
    pooled and per-token entry points."""
    from indecis_b200 import synthetic as S
    cfg = S.tiny(layers=4, hidden=hidden, heads=heads, intermediate=384, vocab=3000)
    om, gm, _ = _models(cfg, seed=7, gamma_noise=0.1)
    _, offs = S.ids_varlen(37, 1, 128, cfg["vocab"], seed=33)
    lens = list(np.diff(offs))
    lens[5] = 0
    lens[20] = 128
    lens[-1] = 127
    offs = np.concatenate([[0], np.cumsum(lens)]).astype(np.int64)
    ids = np.random.default_rng(4).integers(4, cfg["vocab"], int(offs[-1])).astype(np.int32)
    assert np.array_equal(_bits(gm.EncodeTokens((ids, offs))), _bits(om.encode(ids, offs, mode=1, threads=8)))
    assert np.array_equal(_bits(gm.EncodeSeqs((ids, offs))), _bits(om.encode(ids, offs, threads=8)))
    ids2, offs2 = S.ids_fixed(9, 128, cfg["vocab"], seed=34)
    assert np.array_equal(_bits(gm.EncodeSeqs((ids2, offs2))), _bits(om.encode(ids2, offs2, threads=8)))
    gm.close()


def test_batch_composition_and_threads(tiny):
    """concurrency_test.go:12: a sequence's result is the same alone, in any
    batch, and under concurrent calls on one shared model."""
    from indecis_b200 import synthetic as S
    cfg, om, gm, _ = tiny
    ids, offs = S.ids_varlen(12, 3, 150, cfg["vocab"], seed=8)
    seqs = [ids[offs[i]:offs[i + 1]] for i in range(len(offs) - 1)]
    full = gm.EncodeSeqs(seqs)
    for i in (0, 5, 11):
        alone = gm.EncodeSeqs([seqs[i]])
        assert np.array_equal(_bits(alone[0]), _bits(full[i]))
    results = [None] * 8
    def work(t):
        order = list(range(len(seqs)))[t % 3:] + list(range(len(seqs)))[:t % 3]
        out = gm.EncodeSeqs([seqs[j] for j in order])
        results[t] = out[np.argsort(order)]
    ths = [threading.Thread(target=work, args=(t,)) for t in range(8)]
    [t.start() for t in ths]
    [t.join() for t in ths]
    for r in results:
        assert np.array_equal(_bits(r), _bits(full))


def test_edge_cases(tiny):
    from indecis_b200.model import ModernBertError
    cfg, om, gm, _ = tiny
    # empty batch, empty sequences (pooled rows stay zero), one-token sequence
    assert gm.EncodeSeqs([]).shape == (0, cfg["hidden"])
    out = gm.EncodeSeqs([[], [5], []])
    ref = om.encode(np.array([5], np.int32), np.array([0, 0, 1, 1], np.int64))
    assert np.array_equal(_bits(out), _bits(ref))
    assert not out[0].any() and not out[2].any()
    # out-of-vocabulary ids are an error with the reference's wording (infer.go:310-312)
    with pytest.raises(ModernBertError, match="modernbert: id 1000 out of vocabulary"):
        gm.EncodeSeqs([[1, 2, 1000]])
    with pytest.raises(ModernBertError, match="modernbert: id -1 out of vocabulary"):
        gm.EncodeSeqs([[-1]])
    # the model is still usable after the error
    assert np.array_equal(_bits(gm.EncodeSeqs([[5]])), _bits(ref[1:2]))


def test_cls_pooling(igdev, oracle_lib):
    from indecis_b200 import synthetic as S
    cfg = S.tiny(layers=2, vocab=300, pooling="cls")
    om, gm, _ = _models(cfg)
    ids, offs = S.ids_varlen(4, 1, 70, cfg["vocab"], seed=9)
    assert np.array_equal(_bits(gm.EncodeSeqs((ids, offs))), _bits(om.encode(ids, offs)))


def test_head_logits(tiny):
    """heads.go:62-74 in float64 over the pooled vector and per token."""
    import oracle
    from indecis_b200 import synthetic as S
    from indecis_b200.model import Head
    cfg, om, gm, _ = tiny
    heads = [Head(h["name"], h["kind"], h["w"], h["b"] + np.float32(0.01)) for h in S.heads(cfg["hidden"])]
    gm.SetHeads(heads)
    ids, offs = S.ids_varlen(6, 2, 90, cfg["vocab"], seed=10)
    logits, _ = gm.Logits((ids, offs))
    pooled = om.encode(ids, offs)
    tokens = om.encode(ids, offs, mode=1)
    for h, z in zip(heads, logits):
        ref = oracle.head_logits(h.w, h.b, tokens if h.kind == "spans" else pooled)
        assert np.abs(z - ref).max() <= 1e-4
        assert np.array_equal(z, ref)
    a = heads[2].answer(logits[2][0])
    assert abs(sum(a["Probs"].values()) - 1) < 1e-12


def test_head_logits_many(tiny):
    """The per-token and pooled heads over enough tokens and sequences for
    the block-wide float64 kernel (300 sequences, about 6000 tokens)."""
    import oracle
    from indecis_b200 import synthetic as S
    from indecis_b200.model import Head
    cfg, om, gm, _ = tiny
    heads = [Head(h["name"], h["kind"], h["w"], h["b"] - np.float32(0.02)) for h in S.heads(cfg["hidden"], seed=4)]
    gm.SetHeads(heads)
    ids, offs = S.ids_varlen(300, 1, 40, cfg["vocab"], seed=12)
    logits, _ = gm.Logits((ids, offs))
    pooled = om.encode(ids, offs, threads=8)
    tokens = om.encode(ids, offs, mode=1, threads=8)
    for h, z in zip(heads, logits):
        ref = oracle.head_logits(h.w, h.b, tokens if h.kind == "spans" else pooled)
        assert np.array_equal(z, ref), h.name


def test_host_staged_outputs_match_device(igdev):
    """A host call with large outputs copies them out through pinned staging
    in pieces, several host threads moving each piece on; its logits, pooled
    rows and token states equal the device call's bit for bit (ragged
    lengths and empty sequences included), and so do repeated calls."""
    import torch
    from indecis_b200 import _capi
    from indecis_b200 import synthetic as S
    from indecis_b200.model import Config, Head, Model
    gm = Model.from_arrays(Config.from_dict(S.C1), S.weights(S.C1, seed=42))
    heads = [Head(h["name"], h["kind"], h["w"], h["b"]) for h in S.heads(S.C1["hidden"])]
    gm.SetHeads(heads)
    rng = np.random.default_rng(8)
    lens = rng.integers(1, 200, 700)
    lens[[0, 1, 349, 350, 351, 699]] = 0
    offs = np.zeros(len(lens) + 1, np.int64)
    offs[1:] = np.cumsum(lens)
    ids = rng.integers(4, S.C1["vocab"], int(offs[-1])).astype(np.int32)
    assert offs[-1] * 9 * 8 >= 4 << 20  # token logits staged in several pieces
    seqs = [ids[offs[i]:offs[i + 1]] for i in range(len(lens))]
    host, _ = gm.Logits(seqs)
    again, _ = gm.Logits(seqs)
    for a, b in zip(host, again):
        assert np.array_equal(a.view(np.uint64), b.view(np.uint64))
    L = _capi.load()
    pr = sum(h.rows for h in heads if h.kind != "spans")
    tr = sum(h.rows for h in heads if h.kind == "spans")
    d_ids = torch.from_numpy(ids).cuda()
    d_z = torch.empty((len(lens), pr), dtype=torch.float64, device="cuda")
    d_zt = torch.empty((int(offs[-1]), tr), dtype=torch.float64, device="cuda")
    st = torch.cuda.current_stream()
    _capi.check(L.ig_logits_device(gm._h, d_ids.data_ptr(), offs.ctypes.data, len(lens), d_z.data_ptr(),
                                   d_zt.data_ptr(), st.cuda_stream))
    torch.cuda.synchronize()
    z, zt = d_z.cpu().numpy(), d_zt.cpu().numpy()
    po = to = 0
    for h, got in zip(heads, host):
        if h.kind == "spans":
            assert np.array_equal(got.view(np.uint64), zt[:, to:to + h.rows].view(np.uint64)), h.name
            to += h.rows
        else:
            assert np.array_equal(got.view(np.uint64), z[:, po:po + h.rows].view(np.uint64)), h.name
            po += h.rows
    for mode, rows in ((_capi.IG_MODE_POOLED, len(lens)), (_capi.IG_MODE_TOKENS, int(offs[-1]))):
        d_out = torch.empty((rows, S.C1["hidden"]), dtype=torch.float32, device="cuda")
        _capi.check(L.ig_encode_device(gm._h, d_ids.data_ptr(), offs.ctypes.data, len(lens), mode,
                                       d_out.data_ptr(), st.cuda_stream))
        torch.cuda.synchronize()
        got = gm.EncodeSeqs(seqs) if mode == _capi.IG_MODE_POOLED else gm.EncodeTokens(seqs)
        got = np.concatenate(got) if isinstance(got, list) else got
        assert np.array_equal(_bits(got), _bits(d_out.cpu().numpy())), mode
    gm.close()


@pytest.mark.parametrize("lanes", [16, 32])
def test_simd_lanes_bitexact(igdev, oracle_lib, lanes):
    """ExpShift and LayerNorm at 16 and 32 float32 lanes (an AVX-512 or wider
    reference build): the softmax's scalar tail then holds up to lanes - 1
    keys per row, spanning several 16-key chunks of the attention kernels;
    short and long, local and global sequences, bit-exact."""
    from indecis_b200 import synthetic as S
    cfg = S.tiny(layers=3, hidden=256, heads=4, intermediate=384, vocab=1000)
    cfg["V"] = lanes
    om, gm, _ = _models(cfg, seed=7)
    ids, offs = S.ids_varlen(12, 1, 300, cfg["vocab"], seed=lanes)
    assert np.array_equal(_bits(gm.EncodeSeqs((ids, offs))), _bits(om.encode(ids, offs)))
    assert np.array_equal(_bits(gm.EncodeTokens((ids, offs))), _bits(om.encode(ids, offs, mode=1)))
    gm.close()


def test_window_logits_chunked_tail(igdev):
    """Spans windows at a size whose final norm and per-token heads run in
    row chunks with overlapped copies give the same logits as the same
    windows encoded a few at a time (unchunked)."""
    from indecis_b200 import spans as SP
    from indecis_b200 import synthetic as S
    from indecis_b200.model import Config, Head, Model
    gm = Model.from_arrays(Config.from_dict(S.C1), S.weights(S.C1, seed=42))
    gm.SetHeads([Head(h["name"], h["kind"], h["w"], h["b"]) for h in S.heads(S.C1["hidden"])])
    rng = np.random.default_rng(5)
    texts = [rng.integers(4, S.C1["vocab"], int(n)).tolist() for n in rng.integers(200, 2000, 40)]
    big = SP.infer_windows(gm, texts, [2], [1], 128)
    small = SP.infer_windows(gm, texts, [2], [1], 128, batch_size=8)
    assert sum(len(t) for t in texts) >= 16384
    for a, b in zip(big, small):
        for x, y in zip(a.pooled + a.tokens, b.pooled + b.tokens):
            if x is None:
                assert y is None
            else:
                assert np.array_equal(np.asarray(x).view(np.uint64), np.asarray(y).view(np.uint64))
    gm.close()


def test_nonfinite_embedding_rows(igdev, oracle_lib):
    """An embedding table holding a NaN row and a row with an infinity: the
    reference's row quantization sees no finite maximum in the normalized
    NaN rows and turns them into zero rows with scale 0, so the attention and
    MLP inputs stay finite while the residual stream of those tokens carries
    NaN to the end. Every pooled and per-token output bit as the oracle's,
    NaN where it has NaN."""
    from indecis_b200 import synthetic as S
    cfg = S.tiny(layers=3, hidden=256, heads=4, intermediate=384, vocab=800)
    W = S.weights(cfg, seed=23, gamma_noise=0.1)
    W["emb"][7, :] = np.nan
    W["emb"][9, 40] = np.inf
    import oracle
    from indecis_b200.model import Config, Model
    om, gm = oracle.Model(cfg, W), Model.from_arrays(Config.from_dict(cfg), W)
    ids, offs = S.ids_varlen(6, 3, 140, cfg["vocab"], seed=31)
    ids[2], ids[int(offs[3]) + 1], ids[-1] = 7, 9, 7
    for mode, got in ((0, gm.EncodeSeqs((ids, offs))), (1, gm.EncodeTokens((ids, offs)))):
        ref = om.encode(ids, offs, mode=mode, threads=8)
        assert np.isnan(ref).any()
        assert np.array_equal(np.isnan(got), np.isnan(ref)), mode
        ok = ~np.isnan(ref)
        assert np.array_equal(_bits(got)[ok], _bits(ref)[ok]), mode
    gm.close()
