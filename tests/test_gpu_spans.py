"""The Spans branch of infer (spans.go:385-461) on the device: texts longer
than the model cut into windows, each framed by the template's special
tokens and encoded, the pooled heads read from the mean of the first
window's rows, every token's span logits from the window that keeps it.
Bit-exact against the oracle encoder driven through the oracle's window
plan; then the passages decoded from those logits equal the oracle's."""
import json
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "bekko_offsets.jsonl")


def _setup(pooling="mean", seed=21):
    import oracle
    from indecis_b200 import synthetic as S
    from indecis_b200.model import Config, Head, Model
    cfg = S.tiny(layers=3, hidden=128, heads=2, intermediate=192, vocab=700, pooling=pooling)
    W = S.weights(cfg, seed=seed, gamma_noise=0.1)
    gm = Model.from_arrays(Config.from_dict(cfg), W)
    hs = [Head(h["name"], h["kind"], h["w"], h["b"] + np.float32(0.01)) for h in S.heads(cfg["hidden"], seed=seed)]
    gm.SetHeads(hs)
    return cfg, oracle.Model(cfg, W), gm, hs


def _texts(vocab, rng):
    recs = [json.loads(line) for line in open(GOLDEN, encoding="utf-8")]
    texts = [np.asarray(r["ids"], np.int64) % vocab for r in recs[:12]]
    texts += [rng.integers(0, vocab, n) for n in (0, 1, 37, 38, 39, 150, 301)]
    return recs[:12], texts


@pytest.mark.parametrize("pooling", ["mean", "cls"])
def test_infer_windows_bitexact(igdev, oracle_lib, pooling):
    from indecis_b200 import spans as SP
    from oracle import spans as OS
    cfg, om, gm, hs = _setup(pooling)
    rng = np.random.default_rng(4)
    _, texts = _texts(cfg["vocab"], rng)
    prefix, suffix, max_len = [2], [1], 40  # windows of 38 tokens, margins of 2
    heads = [(h.w, h.b, h.kind == "spans") for h in hs]
    want = OS.infer_windows(om, heads, texts, prefix, suffix, max_len)
    for bs in (0, 1, 5):
        got = SP.infer_windows(gm, texts, prefix, suffix, max_len, batch_size=bs)
        for (wp, wt), g in zip(want, got):
            for hi, h in enumerate(hs):
                if h.kind == "spans":
                    assert g.pooled[hi] is None
                    assert np.array_equal(g.tokens[hi].view(np.uint64), wt[hi].view(np.uint64))
                else:
                    assert g.tokens[hi] is None
                    assert np.array_equal(g.pooled[hi].view(np.uint64), wp[hi].view(np.uint64))


def test_decide_spans_on_device_logits(igdev, oracle_lib):
    """answerSpans on the device's token logits, at a temperature and a bias,
    against the oracle's decoding of the oracle's logits."""
    from indecis_b200 import spans as SP
    from oracle import spans as OS
    cfg, om, gm, hs = _setup("mean", seed=5)
    rng = np.random.default_rng(8)
    recs, texts = _texts(cfg["vocab"], rng)
    heads = [(h.w, h.b, h.kind == "spans") for h in hs]
    si = [i for i, h in enumerate(hs) if h.kind == "spans"][0]
    want = OS.infer_windows(om, heads, texts[:len(recs)], [2], [1], 24)
    got = SP.infer_windows(gm, texts[:len(recs)], [2], [1], 24, batch_size=4)
    opts = ["PER", "LOC", "ORG", "MISC"]
    nspans = 0
    for rec, (wp, wt), g in zip(recs, want, got):
        z = g.tokens[si]
        for T, bias in ((1.0, 0.0), (0.05, 0.0), (0.2, 1.5)):
            a = SP.answer_spans(opts, rec["text"], rec["offsets"], z, T, bias)
            logp = [OS.log_softmax(list(r), T) for r in wt[si]]
            o, _ = OS.decode_spans(len(opts), rec["text"].encode(), rec["offsets"], logp, bias)
            assert [(opts[k], s, e, c) for k, s, e, c in o] == [(x.Type, x.Start, x.End, x.Confidence) for x in a]
            nspans += len(a)
    assert nspans > 0


def test_infer_windows_errors(igdev):
    from indecis_b200 import spans as SP
    from indecis_b200.model import ModernBertError
    from indecis_b200 import _capi
    cfg, om, gm, hs = _setup()
    with pytest.raises(ModernBertError, match="out of vocabulary"):
        SP.infer_windows(gm, [[1, 2, 700]], [2], [1], 40)
    with pytest.raises(_capi.IgError):
        SP.infer_windows(gm, [[1, 2]], [2], [1], 0)
    assert SP.infer_windows(gm, [], [2], [1], 40) == []


def test_device_viterbi_matches_host(igdev):
    """The tags decoded on the device (ig_spans_tags: one warp per text) equal
    the host's Viterbi pass, and the passages extracted from them equal
    answer_spans, over many texts at once (real tokenizations, random logits,
    temperatures and a bias)."""
    from indecis_b200 import spans as SP
    recs = [json.loads(line) for line in open(GOLDEN, encoding="utf-8")]
    rng = np.random.default_rng(31)
    opts = ["PER", "LOC", "ORG", "MISC"]
    zs = [rng.standard_normal((len(r["ids"]), 9)) * 3 for r in recs]
    zs += [rng.standard_normal((n, 9)) * 3 for n in (1, 2, 500, 0)]
    for T, bias in ((1.0, 0.0), (0.3, 0.7), (2.0, -0.4)):
        dev = SP.spans_tags(zs, T, bias)
        for z, tags in zip(zs, dev):
            n = z.shape[0]
            if n == 0:
                assert len(tags) == 0
                continue
            logp = np.stack([SP.log_softmax(z[t], T) for t in range(n)])
            text = "x" * n
            offs = [[i, i + 1] for i in range(n)]
            _, host = SP.decode_spans(opts, text, offs, logp, bias, with_tags=True)
            assert np.array_equal(tags, host)
        for r, z, tags in zip(recs, zs, dev):
            assert SP.spans_from_tags(opts, r["text"], r["offsets"], z, tags, T) == \
                SP.answer_spans(opts, r["text"], r["offsets"], z, T, bias)
