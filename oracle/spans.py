"""CPU restatement of the reference's Spans path (TEST INFRASTRUCTURE).

Pure Python, for the small cases the tests build: window planning, tempered
log-softmax, the BIO Viterbi pass and the passage extraction of spans.go,
with the BIO labelling of training (tagTokens) that the round-trip tests use
to build certain tag sequences. Texts are bytes and offsets byte offsets, as
Go strings are. Only tests/ import this module.

Parity: pinned by the reference's own spans tests restated in
tests/test_spans.py (the bias and consistency cases with their values, the
window-plan properties) and by token offsets of the reference's tokenizer
fixture (tests/golden/bekko_offsets.jsonl). Go's math.Exp and math.Log are
not bit-reproduced (Python's libm stands in, within an ulp): decisions are
identical except for scores tied to the last bit.
"""
from __future__ import annotations

import math

import numpy as np

# unicode.IsSpace: Latin-1 spaces, then the White_Space property.
_SPACE = {0x09, 0x0A, 0x0B, 0x0C, 0x0D, 0x20, 0x85, 0xA0, 0x1680, 0x2028, 0x2029, 0x202F, 0x205F, 0x3000}
_SPACE |= set(range(0x2000, 0x200B))
OPEN_PUNCT = "([{«‹“‘\"'¿¡"  # spans.go:287
CLOSE_PUNCT = ",;:!?)]}»›”’\"'"  # spans.go:288
PAIRS = {")": "(", "]": "[", "}": "{", "»": "«", "›": "‹", "”": "“"}  # spans.go:284
RUNE_ERROR = "�"


def is_space(r: str) -> bool:
    return ord(r) in _SPACE


def decode_rune(b: bytes) -> tuple[str, int]:
    """utf8.DecodeRune: the one well-formed rune b starts with, else (U+FFFD, 1)."""
    if not b:
        return RUNE_ERROR, 0
    for k in range(1, 5):
        try:
            s = b[:k].decode("utf-8")
        except UnicodeDecodeError:
            continue
        if len(s) == 1:
            return s, k
    return RUNE_ERROR, 1


def decode_last_rune(b: bytes) -> tuple[str, int]:
    """utf8.DecodeLastRune: the one well-formed rune b ends with, else (U+FFFD, 1)."""
    if not b:
        return RUNE_ERROR, 0
    for k in range(1, 5):
        if k > len(b):
            break
        try:
            s = b[len(b) - k:].decode("utf-8")
        except UnicodeDecodeError:
            continue
        if len(s) == 1:
            return s, k
    return RUNE_ERROR, 1


def is_inside(tag: int) -> bool:
    """spans.go:127."""
    return tag > 0 and tag % 2 == 0


def tag_type(tag: int) -> int:
    """spans.go:126 (Go's truncating division)."""
    return int((tag - 1) / 2)


def plan_windows(n: int, size: int, margin: int):
    """planWindows (spans.go:322-334) -> [(start, end, keep_from, keep_to)]."""
    if n <= size:
        return [(0, n, 0, n)]
    margin = min(margin, (size - 1) // 4)
    k = (n + size - 2 * margin - 1) // (size - 2 * margin)
    out = []
    for i in range(k):
        lo, hi = i * n // k, (i + 1) * n // k
        out.append((max(lo - margin, 0), min(hi + margin, n), lo, hi))
    return out


def log_softmax(z, temperature: float = 1.0) -> list[float]:
    """logSoftmax (spans.go:293-311)."""
    if temperature <= 0:
        temperature = 1
    mx = -math.inf
    for v in z:
        x = v / temperature
        mx = math.nan if math.isnan(mx) or math.isnan(x) else max(mx, x)
    s = 0.0
    for v in z:
        s += math.exp(v / temperature - mx)
    lse = mx + math.log(s) if s > 0 else -math.inf if s == 0 else math.nan
    return [v / temperature - lse for v in z]


def viterbi(logp, bias: float = 0.0) -> list[int]:
    """The tag sequence of decodeSpans (spans.go:172-220)."""
    n = len(logp)
    if n == 0:
        return []
    C = len(logp[0])

    def score(t, c):
        return logp[t][c] + bias if c > 0 else logp[t][c]

    def allowed(p, c):
        return not is_inside(c) or (p > 0 and tag_type(p) == tag_type(c))

    cur = [-math.inf if is_inside(c) else score(0, c) for c in range(C)]
    back = [None] * n
    for t in range(1, n):
        back[t] = [0] * C
        nxt = [0.0] * C
        for c in range(C):
            best, arg = -math.inf, 0
            for p in range(C):
                if allowed(p, c) and cur[p] > best:
                    best, arg = cur[p], p
            nxt[c] = best + score(t, c)
            back[t][c] = arg
        cur = nxt
    tags = [0] * n
    for c in range(C):
        if cur[c] > cur[tags[n - 1]]:
            tags[n - 1] = c
    for t in range(n - 1, 0, -1):
        tags[t - 1] = back[t][tags[t]]
    return tags


def token_core(text: bytes, o) -> tuple[int, int]:
    """tokenCore (spans.go:131-144)."""
    s, e = o
    while s < e:
        r, size = decode_rune(text[s:e])
        if not is_space(r):
            break
        s += size
    if s == e:
        return o[0], o[1]
    return s, e


def _paired(span: bytes, closing: str) -> bool:
    """paired (spans.go:276-282)."""
    op = PAIRS.get(closing)
    if op is None:
        return False
    return span.count(op.encode()) > span.count(closing.encode())


def trim_punct(text: bytes, start: int, end: int) -> tuple[int, int]:
    """trimPunct (spans.go:252-272)."""
    s, e = start, end
    while s < e:
        r, size = decode_rune(text[s:e])
        if r not in OPEN_PUNCT and not is_space(r):
            break
        s += size
    while s < e:
        r, size = decode_last_rune(text[s:e])
        if not is_space(r) and (r not in CLOSE_PUNCT or _paired(text[s:e - size], r)):
            break
        e -= size
    if s == e:
        return start, end
    return s, e


def decode_spans(ntypes: int, text: bytes, offs, logp, bias: float = 0.0):
    """decodeSpans (spans.go:172-246) -> [(type, start, end, confidence)], tags."""
    tags = viterbi(logp, bias)
    n = len(tags)
    out = []
    t = 0
    while t < n:
        if tags[t] == 0:
            t += 1
            continue
        k = tag_type(tags[t])
        start, _ = token_core(text, offs[t])
        end = offs[t][1]
        conf = math.exp(logp[t][tags[t]])
        u = t + 1
        while u < n and is_inside(tags[u]):
            end = offs[u][1]
            conf += math.exp(logp[u][tags[u]])
            u += 1
        start, end = trim_punct(text, start, end)
        assert k < ntypes
        out.append((k, start, end, conf / (u - t)))
        t = u
    return out, tags


def tag_tokens(text: bytes, offs, spans) -> list[int]:
    """tagTokens (spans.go:148-168): spans [(start, end, k)] sorted by start."""
    tags = [0] * len(offs)
    j, prev = 0, -1
    for i, o in enumerate(offs):
        s, e = token_core(text, o)
        while j < len(spans) and spans[j][1] <= s:
            j += 1
        if j < len(spans) and spans[j][0] < e and s < e:
            tags[i] = 2 + 2 * spans[j][2] if prev == j else 1 + 2 * spans[j][2]
            prev = j
            continue
        prev = -1
    return tags


def mean_rows(rows: np.ndarray) -> np.ndarray:
    """meanRows (spans.go:464-477): float64 sums in token order."""
    n, H = rows.shape
    acc = np.zeros(H, np.float64)
    for t in range(n):
        acc += rows[t].astype(np.float64)
    return (acc / float(max(n, 1))).astype(np.float32)


def infer_windows(model, heads, texts, prefix, suffix, max_len: int):
    """The Spans branch of infer (spans.go:385-461) on the oracle encoder:
    heads [(w, b, per_token)]; returns per text ([pooled logits or None per
    head], [token logits or None per head])."""
    from . import head_logits
    prefix, suffix = list(prefix), list(suffix)
    size = max(max_len - len(prefix) - len(suffix), 1)
    out = []
    for ids in texts:
        ids = list(ids)
        pooled = [None] * len(heads)
        tokens = [np.zeros((len(ids), w.shape[0])) if pt else None for (w, b, pt) in heads]
        for (ws, we, kf, kt) in plan_windows(len(ids), size, size // 16):
            seq = np.asarray(prefix + ids[ws:we] + suffix, np.int32)
            states = model.encode(seq, np.asarray([0, len(seq)], np.int64), mode=1)
            if ws == 0:
                x = mean_rows(states)[None, :]
                for hi, (w, b, pt) in enumerate(heads):
                    if not pt:
                        pooled[hi] = head_logits(w, b, x)[0]
            rows = states[len(prefix) + kf - ws:len(prefix) + kt - ws]
            for hi, (w, b, pt) in enumerate(heads):
                if pt and len(rows):
                    tokens[hi][kf:kt] = head_logits(w, b, rows)
        out.append((pooled, tokens))
    return out
