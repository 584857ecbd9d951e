"""Spans questions (spans.go): passages of a text found by BIO tagging.

A Spans head reads every token state and gives the logits of 1 + 2·types
tags (0 outside, 1 + 2k begins a passage of type k, 2 + 2k continues it).
Texts longer than the model are read in overlapping windows; the Viterbi
pass picks the most probable consistent tag sequence and its passages come
back as byte offsets into the text, like the reference's Go strings.

Everything here calls the C ABI: the window planning, log-softmax and
decoding are the library's host code, the encoder and heads its device code.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import numpy as np

from . import _capi

MAX_SPAN_TYPES = 63  # MaxSpanTypes, spans.go:121: a token's tag fits a signed byte


def span_tag_count(types: int) -> int:
    """spanTagCount (spans.go:125)."""
    return 1 + 2 * types


@dataclass
class Span:
    """A passage found by a Spans question: text[Start:End] (Span, spans.go:43-50)."""
    Type: str
    Start: int
    End: int
    Text: str
    Confidence: float


@dataclass
class Window:
    """Tokens [start, end) read in one pass; [keep_from, keep_to) tagged from it (spans.go:314)."""
    start: int
    end: int
    keep_from: int
    keep_to: int


def _text_bytes(text) -> bytes:
    return text.encode("utf-8", "surrogateescape") if isinstance(text, str) else bytes(text)


def plan_windows(n: int, size: int, margin: int) -> list[Window]:
    """planWindows (spans.go:322-334)."""
    L = _capi.load()
    cnt = C.c_int32()
    _capi.check(L.ig_plan_windows(n, size, margin, None, 0, C.byref(cnt)))
    ws = (_capi.IgWindow * cnt.value)()
    _capi.check(L.ig_plan_windows(n, size, margin, ws, cnt.value, C.byref(cnt)))
    return [Window(w.start, w.end, w.keep_from, w.keep_to) for w in ws]


def log_softmax(z, temperature: float = 1.0) -> np.ndarray:
    """logSoftmax (spans.go:293-311)."""
    z = np.ascontiguousarray(z, np.float64)
    out = np.empty_like(z)
    _capi.check(_capi.load().ig_log_softmax(z.ctypes.data, z.size, float(temperature), out.ctypes.data))
    return out


def _offsets(offsets, ntok: int) -> np.ndarray:
    o = np.ascontiguousarray(offsets, np.int32).reshape(-1, 2) if ntok else np.zeros((0, 2), np.int32)
    if o.shape[0] != ntok:
        raise ValueError(f"{o.shape[0]} offsets for {ntok} tokens")
    return o


def _spans(options, tb: bytes, found, n: int) -> list[Span]:
    out = []
    for s in found[:n]:
        out.append(Span(options[s.type], s.start, s.end, tb[s.start:s.end].decode("utf-8", "surrogateescape"),
                        s.confidence))
    return out


def decode_spans(options, text, offsets, logp, bias: float = 0.0, with_tags: bool = False):
    """decodeSpans (spans.go:172-246): logp [tokens][tags] log-probabilities,
    offsets [tokens][2] byte ranges. Returns the passages (and the tags)."""
    logp = np.ascontiguousarray(logp, np.float64)
    ntok = logp.shape[0] if logp.ndim == 2 else 0
    ntags = logp.shape[1] if logp.ndim == 2 and ntok else span_tag_count(len(options))
    o = _offsets(offsets, ntok)
    tb = _text_bytes(text)
    tags = np.zeros(ntok, np.int32)
    found = (_capi.IgSpan * max(ntok, 1))()
    n = C.c_int32()
    _capi.check(_capi.load().ig_decode_spans(logp.ctypes.data, ntok, ntags, float(bias), tb, len(tb), o.ctypes.data,
                                             tags.ctypes.data, found, ntok, C.byref(n)))
    spans = _spans(options, tb, found, n.value)
    return (spans, tags) if with_tags else spans


def answer_spans(options, text, offsets, z, temperature: float = 1.0, bias: float = 0.0) -> list[Span]:
    """answerSpans (spans.go:479-491): each token's logits z [tokens][tags]
    through logSoftmax at the head's temperature, then decodeSpans."""
    z = np.ascontiguousarray(z, np.float64)
    ntok = z.shape[0] if z.ndim == 2 else 0
    ntags = z.shape[1] if ntok else span_tag_count(len(options))
    o = _offsets(offsets, ntok)
    tb = _text_bytes(text)
    found = (_capi.IgSpan * max(ntok, 1))()
    n = C.c_int32()
    _capi.check(_capi.load().ig_answer_spans(z.ctypes.data, ntok, ntags, ntags, float(temperature), float(bias), tb,
                                             len(tb), o.ctypes.data, found, ntok, C.byref(n)))
    return _spans(options, tb, found, n.value)


@dataclass
class Inference:
    """What the model computed for one text (inference, spans.go:362-367):
    per head, the pooled logits (None for Spans heads) or the logits of every
    token of the text (None for the other heads)."""
    pooled: list = field(default_factory=list)
    tokens: list = field(default_factory=list)


def infer_windows(model, texts, prefix, suffix, max_len: int, batch_size: int = 0) -> list[Inference]:
    """The Spans branch of infer (spans.go:385-461) on tokenized texts (each
    a sequence of token ids without the template's special tokens): windows
    of max(max_len - |prefix| - |suffix|, 1) tokens framed by prefix and
    suffix, encoded on the device batch_size windows at a time (0: all)."""
    from .model import ModernBertError, _concat
    ids, offs = _concat([np.asarray(t, np.int32) for t in texts])
    ninp = len(offs) - 1
    pre = np.ascontiguousarray(prefix, np.int32)
    suf = np.ascontiguousarray(suffix, np.int32)
    L = _capi.load()
    pr, tr = C.c_int32(), C.c_int32()
    _capi.check(L.ig_model_head_rows(model._h, C.byref(pr), C.byref(tr)))
    z = np.zeros((ninp, pr.value), np.float64)
    zt = np.zeros((int(offs[-1]), tr.value), np.float64)
    rc = L.ig_infer_windows(model._h, ids.ctypes.data, offs.ctypes.data, ninp, pre.ctypes.data, len(pre),
                            suf.ctypes.data, len(suf), int(max_len), int(batch_size), z.ctypes.data, z.size,
                            zt.ctypes.data, zt.size)
    if rc == _capi.IG_ERR_OUT_OF_VOCAB:
        raise ModernBertError(_capi.last_error())
    _capi.check(rc)
    out = []
    for i in range(ninp):
        inf, po, to = Inference(), 0, 0
        for h in model.heads:
            if h.kind == "spans":
                inf.pooled.append(None)
                inf.tokens.append(zt[offs[i]:offs[i + 1], to:to + h.rows])
                to += h.rows
            else:
                inf.pooled.append(z[i, po:po + h.rows])
                inf.tokens.append(None)
                po += h.rows
        out.append(inf)
    return out


def spans_tags(zs, temperature: float = 1.0, bias: float = 0.0, device: int = 0):
    """The tags of answer_spans for many texts at once, decoded on the device
    (ig_spans_tags: log-softmax and Viterbi, one warp per text). zs: per text
    its logits [tokens][tags]. Returns one int32 array of tags per text."""
    zs = [np.ascontiguousarray(z, np.float64) for z in zs]
    ntags = next((z.shape[1] for z in zs if z.ndim == 2 and z.shape[0]), 1)
    offs = np.zeros(len(zs) + 1, np.int64)
    offs[1:] = np.cumsum([z.shape[0] if z.ndim == 2 else 0 for z in zs])
    flat = np.concatenate([z.reshape(-1, ntags) for z in zs]) if offs[-1] else np.zeros((0, ntags))
    flat = np.ascontiguousarray(flat, np.float64)
    tags = np.zeros(int(offs[-1]), np.int32)
    _capi.check(_capi.load().ig_spans_tags(flat.ctypes.data, ntags, offs.ctypes.data, len(zs), ntags,
                                           float(temperature), float(bias), tags.ctypes.data, device))
    return [tags[offs[i]:offs[i + 1]] for i in range(len(zs))]


def spans_from_tags(options, text, offsets, z, tags, temperature: float = 1.0) -> list[Span]:
    """decodeSpans' passage extraction for a given tag sequence (ig_spans_from_tags)."""
    z = np.ascontiguousarray(z, np.float64)
    ntok = z.shape[0] if z.ndim == 2 else 0
    ntags = z.shape[1] if ntok else span_tag_count(len(options))
    o = _offsets(offsets, ntok)
    t = np.ascontiguousarray(tags, np.int32)
    tb = _text_bytes(text)
    found = (_capi.IgSpan * max(ntok, 1))()
    n = C.c_int32()
    _capi.check(_capi.load().ig_spans_from_tags(z.ctypes.data, ntok, ntags, ntags, float(temperature), t.ctypes.data,
                                                tb, len(tb), o.ctypes.data, found, ntok, C.byref(n)))
    return _spans(options, tb, found, n.value)
