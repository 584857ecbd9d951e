"""The host side of the Spans path through the C ABI, against the oracle's
restatement of spans.go and the reference's own spans tests
(spans_test.go): window plans, log-softmax, the BIO Viterbi decoding and the
passage extraction (token cores, punctuation trimming) on real tokenizations
of the reference's tokenizer fixture. No GPU: these entry points are host
code."""
import itertools
import json
import math
import os

import numpy as np
import pytest

from indecis_b200 import _capi
from indecis_b200 import spans as S
from oracle import spans as O

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "bekko_offsets.jsonl")


def _texts():
    return [json.loads(line) for line in open(GOLDEN, encoding="utf-8")]


# ---- planWindows: TestPlanWindows (spans_test.go:20-53) -------------------

def test_plan_windows_properties():
    for size in (1, 2, 3, 7, 16, 254):
        for margin in (0, size // 16, size // 8, size):
            for n in range(0, 4 * size + 5):
                ws = S.plan_windows(n, size, margin)
                assert [(w.start, w.end, w.keep_from, w.keep_to) for w in ws] == O.plan_windows(n, size, margin)
                nxt = 0
                m = min(margin, (size - 1) // 4)
                for i, w in enumerate(ws):
                    assert w.end - w.start <= size and w.start >= 0 and w.end <= n
                    assert w.keep_from == nxt and w.keep_from >= w.start and w.keep_to <= w.end
                    assert w.keep_to > w.keep_from or n == 0
                    assert not (i > 0 and w.keep_from - w.start < m)
                    assert not (i < len(ws) - 1 and w.end - w.keep_to < m)
                    nxt = w.keep_to
                assert nxt == n
                if n > size:
                    for w in ws[1:]:
                        d = (w.end - w.start) - (ws[0].end - ws[0].start)
                        assert -margin - 1 <= d <= margin + 1


def test_plan_windows_errors():
    import ctypes as C
    L = _capi.load()
    cnt = C.c_int32()
    assert L.ig_plan_windows(10, 0, 0, None, 0, C.byref(cnt)) == _capi.IG_ERR_BAD_ARG
    assert L.ig_plan_windows(-1, 4, 0, None, 0, C.byref(cnt)) == _capi.IG_ERR_BAD_ARG
    ws = (_capi.IgWindow * 1)()
    assert L.ig_plan_windows(100, 10, 1, ws, 1, C.byref(cnt)) == _capi.IG_ERR_BAD_ARG
    assert cnt.value == 13  # the count still comes back


# ---- logSoftmax ------------------------------------------------------------

def test_log_softmax_matches_oracle():
    rng = np.random.default_rng(3)
    for n in (0, 1, 2, 9, 127):
        for T in (1.0, 0.37, 2.5, 0.0, -1.0):
            z = rng.standard_normal(n) * 6
            got = S.log_softmax(z, T)
            want = O.log_softmax(list(z), T)
            assert np.array_equal(got, np.asarray(want, np.float64))
            if n:
                assert abs(math.fsum(np.exp(got)) - 1) < 1e-12
    # -inf logits give zero probability, the rest still normalize.
    got = S.log_softmax([0.0, -math.inf, 1.0])
    assert got[1] == -math.inf and abs(math.exp(got[0]) + math.exp(got[2]) - 1) < 1e-15
    # NaN propagates like Go's max.
    assert np.isnan(S.log_softmax([0.0, math.nan])).all()


# ---- decodeSpans: the reference's cases -----------------------------------

def test_decode_spans_bias():
    """TestDecodeSpansBias (spans_test.go:364-376)."""
    offs = [[0, 4]]
    logp = [[math.log(0.6), math.log(0.3), math.log(0.1)]]
    assert S.decode_spans(["PER"], "Jean", offs, logp, 0) == []
    got = S.decode_spans(["PER"], "Jean", offs, logp, 1)
    assert len(got) == 1 and got[0].Text == "Jean" and abs(got[0].Confidence - 0.3) < 1e-9


def test_decode_spans_consistent():
    """TestDecodeSpansConsistent (spans_test.go:160-218): the decoded path is
    the best allowed tag sequence (brute force)."""
    opts = ["PER", "LOC"]
    text = "a b c"
    offs = [[0, 1], [1, 3], [3, 5]]
    lp = lambda *p: [math.log(v) for v in p]
    logp = [lp(0.30, 0.25, 0.40, 0.03, 0.02), lp(0.10, 0.10, 0.10, 0.10, 0.60), lp(0.90, 0.025, 0.025, 0.025, 0.025)]
    got, tags = S.decode_spans(opts, text, offs, logp, 0, with_tags=True)
    best, best_tags = -math.inf, None
    for seq in itertools.product(range(5), repeat=3):
        ok = not O.is_inside(seq[0])
        for i in range(1, 3):
            ok = ok and (not O.is_inside(seq[i]) or (seq[i - 1] > 0 and O.tag_type(seq[i - 1]) == O.tag_type(seq[i])))
        s = logp[0][seq[0]] + logp[1][seq[1]] + logp[2][seq[2]]
        if ok and s > best:
            best, best_tags = s, list(seq)
    assert list(tags) == best_tags
    want = []
    i = 0
    while i < 3:
        if best_tags[i] == 0:
            i += 1
            continue
        j = i + 1
        while j < 3 and O.is_inside(best_tags[j]):
            j += 1
        start, _ = O.token_core(text.encode(), offs[i])
        want.append((opts[O.tag_type(best_tags[i])], start, offs[j - 1][1]))
        i = j
    assert [(s.Type, s.Start, s.End) for s in got] == want


def test_viterbi_brute_force_random():
    """Random scores, with ties and -inf: the decoded tags score as the best
    allowed sequence, and equal the oracle's (same tie-breaking)."""
    rng = np.random.default_rng(11)
    for trial in range(200):
        n = int(rng.integers(1, 6))
        types = int(rng.integers(1, 3))
        C = 1 + 2 * types
        logp = np.round(rng.standard_normal((n, C)), 1 if trial % 2 else 6)
        if trial % 5 == 0:
            logp[rng.random((n, C)) < 0.2] = -math.inf
        bias = float(rng.choice([0.0, 0.5, -0.3]))
        text = "x" * n
        offs = [[i, i + 1] for i in range(n)]
        _, tags = S.decode_spans([f"T{k}" for k in range(types)], text, offs, logp, bias, with_tags=True)
        assert list(tags) == O.viterbi(logp.tolist(), bias)
        sc = lambda t, c: logp[t][c] + bias if c > 0 else logp[t][c]
        best = -math.inf
        for seq in itertools.product(range(C), repeat=n):
            ok = not O.is_inside(seq[0]) and all(
                not O.is_inside(seq[i]) or (seq[i - 1] > 0 and O.tag_type(seq[i - 1]) == O.tag_type(seq[i]))
                for i in range(1, n))
            if ok:
                best = max(best, sum(sc(t, c) for t, c in enumerate(seq)))
        got = sum(sc(t, int(c)) for t, c in enumerate(tags))
        assert got == best or (math.isinf(best) and math.isinf(got))


# ---- passages on real tokenizations ---------------------------------------

def _gold_spans(rng, text: bytes, offs):
    """Non-overlapping passages whose bounds fall on token cores."""
    n = len(offs)
    spans, t = [], 0
    while t < n:
        if rng.random() < 0.35:
            u = min(n, t + int(rng.integers(1, 4)))
            s, _ = O.token_core(text, offs[t])
            e = offs[u - 1][1]
            if s < e and (not spans or spans[-1][1] <= s):
                spans.append((s, e, int(rng.integers(0, 3))))
            t = u + 1
        else:
            t += 1
    return spans


def test_tag_decode_round_trip_tokenizer_fixture():
    """TestTagDecodeRoundTrip (spans_test.go:98-143) on the reference
    tokenizer's own offsets: certain tags from tagTokens decode to the
    passages (trimmed of edge punctuation), as the oracle decodes them."""
    rng = np.random.default_rng(5)
    opts = ["PER", "LOC", "ORG"]
    C = 1 + 2 * len(opts)
    checked = 0
    for rec in _texts():
        text = rec["text"].encode("utf-8")
        offs = rec["offsets"]
        for _ in range(3):
            gold = _gold_spans(rng, text, offs)
            tags = O.tag_tokens(text, offs, gold)
            logp = np.full((len(tags), C), -30.0)
            logp[np.arange(len(tags)), tags] = 0.0
            got = S.decode_spans(opts, rec["text"], offs, logp)
            want, want_tags = O.decode_spans(len(opts), text, offs, logp.tolist())
            assert want_tags == tags
            assert [(opts[k], s, e, c) for k, s, e, c in want] == [(g.Type, g.Start, g.End, g.Confidence) for g in got]
            for g in got:
                assert g.Text == text[g.Start:g.End].decode("utf-8", "surrogateescape")
                assert g.Confidence == 1.0
            # Passages without edge punctuation come back exactly.
            exact = [(s, e, k) for s, e, k in gold if O.trim_punct(text, s, e) == (s, e)]
            got_set = {(g.Start, g.End, opts.index(g.Type)) for g in got}
            assert set(exact) <= got_set
            checked += len(gold)
    assert checked > 200


@pytest.mark.parametrize("text,lo,hi,want", [
    ("Pascal Lamy, est", 0, 12, "Pascal Lamy"),           # "Lamy," : the comma is not part of the name
    ("(Lyon) x", 0, 6, "Lyon"),
    ("« Marseille »", 0, len("« Marseille »".encode()), "Marseille"),
    ("Mme Roux (née Martin), à", 0, len("Mme Roux (née Martin),".encode()), "Mme Roux (née Martin)"),
    ("J.-P. Sartre", 0, 5, "J.-P."),                      # dots stay
    ("Inc.", 0, 4, "Inc."),
    ("«»", 0, 4, "«»"),                                    # only punctuation: kept whole
    ("  Lyon  ", 0, 8, "Lyon"),
    ("“Quote”", 0, len("“Quote”".encode()), "Quote"),
    ("¿Qué?", 0, len("¿Qué?".encode()), "Qué"),
    ("f(x)", 0, 4, "f(x)"),                                # a bracket closing a pair opened inside
    ("x)", 0, 2, "x"),
])
def test_trim_punct_cases(text, lo, hi, want):
    """trimPunct (spans.go:248-272) through a one-token passage."""
    logp = [[-30.0, 0.0, -30.0]]
    got = S.decode_spans(["T"], text, [[lo, hi]], logp)
    assert len(got) == 1 and got[0].Text == want
    s, e = O.trim_punct(text.encode(), lo, hi)
    assert (got[0].Start, got[0].End) == (s, e)


def test_decode_spans_random_bytes():
    """Invalid UTF-8, unusual spaces and punctuation in random byte strings:
    the library's rune decoding, spaces and trimming agree with the oracle's."""
    rng = np.random.default_rng(17)
    alphabet = [b" ", b"\t", b"\xc2\xa0", b"\xe2\x80\x83", b"\xe3\x80\x80", b"\xc2\x85", b"\x1c", b"a", b"Z",
                b"(", b")", b"\xc2\xab", b"\xc2\xbb", b"\xe2\x80\x9c", b"\xe2\x80\x9d", b",", b".", b"'", b"\"",
                b"\x80", b"\xc3", b"\xe2\x80", b"\xf0\x9f\x98\x80", b"\xed\xa0\x80", b"\xc0\xaf", b"\xff", b"!",
                b"\xc2\xbf", b"\xe2\x80\xba"]
    opts = ["A", "B"]
    for trial in range(400):
        parts = [alphabet[i] for i in rng.integers(0, len(alphabet), int(rng.integers(1, 14)))]
        text = b"".join(parts)
        cuts = sorted(set([0, len(text)] + list(rng.integers(0, len(text) + 1, int(rng.integers(1, 5))))))
        offs = [[a, b] for a, b in zip(cuts, cuts[1:])]
        logp = rng.standard_normal((len(offs), 5))
        for t in range(len(offs)):
            logp[t] = O.log_softmax(list(logp[t] * 3))
        bias = float(rng.choice([0.0, 2.0]))
        got = S.decode_spans(opts, text, offs, logp, bias)
        want, _ = O.decode_spans(2, text, offs, logp.tolist(), bias)
        assert [(opts[k], s, e) for k, s, e, _ in want] == [(g.Type, g.Start, g.End) for g in got], text
        for (k, s, e, c), g in zip(want, got):
            assert g.Confidence == c


def test_answer_spans_is_log_softmax_then_decode():
    """answerSpans (spans.go:479-491) at a temperature."""
    rng = np.random.default_rng(2)
    rec = _texts()[7]
    n = len(rec["ids"])
    z = rng.standard_normal((n, 7)) * 4
    for T, bias in ((1.0, 0.0), (0.6, 0.4), (0.0, -0.2)):
        logp = np.stack([S.log_softmax(z[t], T) for t in range(n)]) if n else np.zeros((0, 7))
        assert S.answer_spans(["a", "b", "c"], rec["text"], rec["offsets"], z, T, bias) == \
            S.decode_spans(["a", "b", "c"], rec["text"], rec["offsets"], logp, bias)


def test_decode_spans_errors():
    import ctypes as C
    L = _capi.load()
    logp = np.array([[-5.0, 0.0, -5.0]])
    offs = np.array([[0, 9]], np.int32)  # beyond a 4-byte text
    n = C.c_int32()
    out = (_capi.IgSpan * 1)()
    assert L.ig_decode_spans(logp.ctypes.data, 1, 3, 0.0, b"Jean", 4, offs.ctypes.data, None, out, 1,
                             C.byref(n)) == _capi.IG_ERR_BAD_ARG
    assert "out of a text of 4 bytes" in _capi.last_error()
    offs = np.array([[0, 4]], np.int32)
    assert L.ig_decode_spans(logp.ctypes.data, 1, 3, 0.0, b"Jean", 4, offs.ctypes.data, None, out, 0,
                             C.byref(n)) == _capi.IG_ERR_BAD_ARG
    assert n.value == 1
    # No tokens: no passages.
    assert S.decode_spans(["PER"], "", [], np.zeros((0, 3))) == []
