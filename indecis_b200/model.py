"""Host-side mirror of indecis' int8 ModernBERT inference API over the C ABI.

Names, argument meanings and errors follow the Go reference:
  internal/modernbert/model.go   Config, FromTensors, validate
  internal/modernbert/infer.go   SetInt8, Encode, EncodeSeqs, EncodeTokens, run
  heads.go                       head.logits / head.answer (noul, choice, score, spans)
The computation runs in libindecis_b200.so on an sm_100 GPU; nothing here
computes the encoder on the CPU.
"""
from __future__ import annotations

import ctypes as C
import math
from dataclasses import dataclass, field

import numpy as np

from . import _capi


class ModernBertError(ValueError):
    """An error the reference returns as a Go `error` (same wording)."""


def _go_quote(s: str) -> str:
    """Go's %q of a printable string: double quotes, backslash escapes."""
    return '"' + s.replace("\\", "\\\\").replace('"', '\\"') + '"'


@dataclass
class Config:
    """modernbert.Config (internal/modernbert/model.go:25-49)."""
    hidden_size: int
    num_hidden_layers: int
    num_attention_heads: int
    intermediate_size: int
    vocab_size: int
    norm_eps: float = 1e-5
    global_attn_every_n_layers: int = 3
    local_attention: int = 128
    global_rope_theta: float = 10000.0
    local_rope_theta: float = 10000.0
    pad_token_id: int = 0
    hidden_activation: str = "gelu"
    classifier_pooling: str = "mean"
    attention_bias: bool = False
    mlp_bias: bool = False
    norm_bias: bool = False
    simd_lanes: int = 8

    @classmethod
    def from_dict(cls, d: dict) -> "Config":
        """From the synthetic-shape dicts (indecis_b200.synthetic) or a config.json."""
        if "hidden" in d:
            return cls(hidden_size=d["hidden"], num_hidden_layers=d["layers"], num_attention_heads=d["heads"],
                       intermediate_size=d["intermediate"], vocab_size=d["vocab"], norm_eps=d["norm_eps"],
                       global_attn_every_n_layers=d["global_every"], local_attention=d["local_attention"],
                       global_rope_theta=d["global_theta"], local_rope_theta=d["local_theta"],
                       classifier_pooling=d.get("pooling", "mean"), simd_lanes=d.get("V", 8))
        keys = {f for f in cls.__dataclass_fields__}
        return cls(**{k: v for k, v in d.items() if k in keys})

    def head_dim(self) -> int:
        return self.hidden_size // self.num_attention_heads

    def is_global(self, l: int) -> bool:
        return l % self.global_attn_every_n_layers == 0

    def window(self) -> int:
        return self.local_attention // 2

    def cls(self) -> bool:
        return self.classifier_pooling == "cls"

    def validate(self):
        """Config.validate (model.go:64-80), same messages."""
        if (self.hidden_size <= 0 or self.num_hidden_layers <= 0 or self.num_attention_heads <= 0
                or self.intermediate_size <= 0 or self.vocab_size <= 0):
            raise ModernBertError("modernbert: invalid dimensions")
        if self.hidden_size % self.num_attention_heads != 0 or self.head_dim() % 2 != 0:
            raise ModernBertError(f"modernbert: hidden_size {self.hidden_size} incompatible with "
                                  f"{self.num_attention_heads} heads")
        if self.global_attn_every_n_layers <= 0 or self.local_attention <= 0:
            raise ModernBertError("modernbert: invalid attention windows")
        if self.hidden_activation != "gelu":
            raise ModernBertError(f"modernbert: activation {_go_quote(self.hidden_activation)} not supported")
        if self.attention_bias or self.mlp_bias or self.norm_bias:
            raise ModernBertError("modernbert: biases are not supported")
        if self.classifier_pooling not in ("", "mean", "cls"):
            raise ModernBertError(f"modernbert: pooling {_go_quote(self.classifier_pooling)} not supported")

    def to_c(self) -> _capi.IgConfig:
        return _capi.IgConfig(vocab=self.vocab_size, hidden=self.hidden_size, layers=self.num_hidden_layers,
                              heads=self.num_attention_heads, intermediate=self.intermediate_size,
                              global_every=self.global_attn_every_n_layers, local_attention=self.local_attention,
                              pooling=1 if self.cls() else 0, norm_eps=self.norm_eps,
                              global_theta=self.global_rope_theta, local_theta=self.local_rope_theta,
                              simd_lanes=self.simd_lanes)


@dataclass
class Batch:
    """modernbert.Batch (internal/modernbert/forward.go:10-15): right-padded."""
    IDs: np.ndarray
    Lens: list
    T: int

    def B(self) -> int:
        return len(self.Lens)


def new_batch(seqs, pad: int = 0) -> Batch:
    """NewBatch (forward.go:17-30)."""
    T = max((len(s) for s in seqs), default=0)
    ids = np.full(len(seqs) * T, pad, np.int32)
    for i, s in enumerate(seqs):
        ids[i * T:i * T + len(s)] = s
    return Batch(ids, [len(s) for s in seqs], T)


def _concat(seqs):
    """seqs -> (ids int32 [N], offs int64 [B+1]) as run() lays them out (infer.go:307-315)."""
    if isinstance(seqs, tuple) and len(seqs) == 2 and isinstance(seqs[1], np.ndarray):
        ids, offs = seqs
        return np.ascontiguousarray(ids, np.int32), np.ascontiguousarray(offs, np.int64)
    lens = [len(s) for s in seqs]
    offs = np.zeros(len(seqs) + 1, np.int64)
    offs[1:] = np.cumsum(lens)
    ids = np.concatenate([np.asarray(s, np.int64) for s in seqs]) if seqs and offs[-1] else np.zeros(0, np.int64)
    if ids.size and (ids.min() < -2**31 or ids.max() >= 2**31):
        bad = int(ids[(ids < -2**31) | (ids >= 2**31)][0])
        raise ModernBertError(f"modernbert: id {bad} out of vocabulary")
    return np.ascontiguousarray(ids, np.int32), offs


_TENSOR_NAMES = {
    "emb": "embeddings.tok_embeddings.weight", "emb_norm": "embeddings.norm.weight",
    "final_norm": "final_norm.weight",
}


class MappedEmbeddings:
    """indecis mappedEmbeddings (embeddings.go:9-68): bf16 rows [vocab][hidden]
    (value = bits << 16) with float32 rows for the ids training modified; or
    an int8 table with a float32 scale per row (newInt8Embeddings). Row gives
    a row on the host; Model.SetEmbeddingTable uploads the table as stored."""

    def __init__(self, hidden: int, bf16=None, exact_ids=None, exact_rows=None, i8=None, scale=None):
        self.h = hidden
        if i8 is not None:
            self.i8 = np.ascontiguousarray(i8, np.int8)
            self.scale = np.ascontiguousarray(scale, np.float32)
            if self.i8.size != len(self.scale) * hidden:
                raise ModernBertError(f"indecis: int8 table of {self.i8.size} bytes for {len(self.scale)} rows")
            self.bf16 = None
            return
        self.i8 = None
        self.bf16 = np.ascontiguousarray(bf16, np.uint16).reshape(-1, hidden)
        ids = np.ascontiguousarray([] if exact_ids is None else exact_ids, np.int32)
        rows = np.ascontiguousarray(np.zeros((0, hidden)) if exact_rows is None else exact_rows, np.float32)
        if rows.size != len(ids) * hidden:
            raise ModernBertError("indecis: malformed exact rows")
        vocab = self.bf16.shape[0]
        self.exact = {}
        for i, r in enumerate(ids.tolist()):
            if r < 0 or r >= vocab:
                raise ModernBertError(f"indecis: exact row {r} out of vocabulary")
            self.exact[r] = i
        self.exact_ids, self.exact_rows = ids, rows.reshape(len(ids), hidden)

    def Row(self, id_: int) -> np.ndarray:
        if self.i8 is not None:
            return (self.i8.reshape(-1, self.h)[id_].astype(np.float32) * self.scale[id_]).astype(np.float32)
        if id_ in self.exact:
            return self.exact_rows[self.exact[id_]].copy()
        return (self.bf16[id_].astype(np.uint32) << 16).view(np.float32)

    def matrix(self) -> np.ndarray:
        """The whole table in float32 (EmbeddingMatrix, infer.go:39-50)."""
        vocab = (self.i8.size // self.h) if self.i8 is not None else self.bf16.shape[0]
        return np.stack([self.Row(i) for i in range(vocab)]).astype(np.float32)


class Model:
    """modernbert.Model restricted to inference on the device. `device` is one
    GPU ordinal, or a list of them: the model is then replicated on each and
    every call's sequences are split across them by cost (no collective)."""

    def __init__(self, cfg: Config, handle, device: int):
        self.Cfg = cfg
        self._h = handle
        self.device = device
        self._int8 = True
        self.heads: list[Head] = []

    # ---- construction (model.go:179-234) ----
    @classmethod
    def FromTensors(cls, cfg: Config, tensors: dict, device: int = 0) -> "Model":
        """Assembles a model from tensors named as in transformers (the "model."
        prefix is accepted) and uploads it; quantization happens on the device."""
        cfg.validate()
        H, I, V, L = cfg.hidden_size, cfg.intermediate_size, cfg.vocab_size, cfg.num_hidden_layers

        def get(name, *shape):
            t = tensors.get(name)
            if t is None:
                t = tensors.get("model." + name)
            if t is None:
                raise ModernBertError(f"modernbert: tensor {name} missing")
            t = np.ascontiguousarray(t, np.float32)
            if list(t.shape) != list(shape):
                raise ModernBertError(f"modernbert: {name}: shape {list(t.shape)}, expected {list(shape)}")
            return t

        keep = [get("embeddings.tok_embeddings.weight", V, H), get("embeddings.norm.weight", H),
                get("final_norm.weight", H)]
        per = {k: [] for k in ("attn_norm", "wqkv", "wo", "mlp_norm", "wi", "wo_mlp")}
        for l in range(L):
            p = f"layers.{l}."
            per["attn_norm"].append(get(p + "attn_norm.weight", H) if l > 0 else None)
            per["wqkv"].append(get(p + "attn.Wqkv.weight", 3 * H, H))
            per["wo"].append(get(p + "attn.Wo.weight", H, H))
            per["mlp_norm"].append(get(p + "mlp_norm.weight", H))
            per["wi"].append(get(p + "mlp.Wi.weight", 2 * I, H))
            per["wo_mlp"].append(get(p + "mlp.Wo.weight", H, I))
        return cls._create(cfg, keep, per, device)

    @classmethod
    def from_arrays(cls, cfg: Config, w: dict, device: int = 0) -> "Model":
        """From the layout of indecis_b200.synthetic.weights (same arrays, short keys)."""
        tensors = {_TENSOR_NAMES[k]: w[k] for k in ("emb", "emb_norm", "final_norm")}
        for l in range(cfg.num_hidden_layers):
            p = f"layers.{l}."
            if l > 0:
                tensors[p + "attn_norm.weight"] = w["attn_norm"][l]
            tensors[p + "attn.Wqkv.weight"] = w["wqkv"][l]
            tensors[p + "attn.Wo.weight"] = w["wo"][l]
            tensors[p + "mlp_norm.weight"] = w["mlp_norm"][l]
            tensors[p + "mlp.Wi.weight"] = w["wi"][l]
            tensors[p + "mlp.Wo.weight"] = w["wo_mlp"][l]
        return cls.FromTensors(cfg, tensors, device)

    @classmethod
    def _create(cls, cfg, keep, per, device):
        L = cfg.num_hidden_layers
        lib = _capi.load()

        def ptrs(name):
            arr = (C.c_void_p * L)(*[0 if a is None else a.ctypes.data for a in per[name]])
            return C.cast(arr, C.POINTER(C.c_void_p)), arr

        hold = {}
        fields = {}
        for name in per:
            fields[name], hold[name] = ptrs(name)
        w = _capi.IgWeights(tok_embeddings=keep[0].ctypes.data, emb_norm=keep[1].ctypes.data,
                            final_norm=keep[2].ctypes.data, **fields)
        c = cfg.to_c()
        h = C.c_void_p()
        if isinstance(device, (list, tuple)):
            devs = (C.c_int32 * len(device))(*device)
            _capi.check(lib.ig_model_create_multi(C.byref(c), C.byref(w), devs, len(device), C.byref(h)))
        else:
            _capi.check(lib.ig_model_create(C.byref(c), C.byref(w), device, C.byref(h)))
        return cls(cfg, h, device)

    @classmethod
    def FromStored(cls, cfg: Config, stored: dict, table: "MappedEmbeddings", device=0) -> "Model":
        """Load's path (model.go:661-735) without decoding on the host: every
        layer tensor goes to the device in its stored dtype and is decoded there
        as safetensors decodes it; the embedding table is uploaded as stored.
        stored maps transformers names to (dtype, raw array): "F32" float32,
        "BF16" / "F16" uint16 bits, "I8" int8."""
        cfg.validate()
        H, I, L = cfg.hidden_size, cfg.intermediate_size, cfg.num_hidden_layers
        lib = _capi.load()
        keep = []

        def view(name, *shape):
            t = stored.get(name, stored.get("model." + name))
            if t is None:
                raise ModernBertError(f"modernbert: tensor {name} missing")
            dt, raw = t
            want = {"F32": np.float32, "BF16": np.uint16, "F16": np.uint16, "I8": np.int8}.get(dt)
            raw = np.ascontiguousarray(raw, want)
            if list(raw.shape) != list(shape):
                raise ModernBertError(f"modernbert: {name}: shape {list(raw.shape)}, expected {list(shape)}")
            keep.append(raw)
            return _capi.IgTensor(dtype=_capi.IG_DT[dt] if isinstance(dt, str) else int(dt), data=raw.ctypes.data)

        per = {k: (_capi.IgTensor * L)() for k in ("attn_norm", "wqkv", "wo", "mlp_norm", "wi", "wo_mlp")}
        for l in range(L):
            p = f"layers.{l}."
            if l > 0:
                per["attn_norm"][l] = view(p + "attn_norm.weight", H)
            per["wqkv"][l] = view(p + "attn.Wqkv.weight", 3 * H, H)
            per["wo"][l] = view(p + "attn.Wo.weight", H, H)
            per["mlp_norm"][l] = view(p + "mlp_norm.weight", H)
            per["wi"][l] = view(p + "mlp.Wi.weight", 2 * I, H)
            per["wo_mlp"][l] = view(p + "mlp.Wo.weight", H, I)
        w = _capi.IgStoredWeights(emb_norm=view("embeddings.norm.weight", H), final_norm=view("final_norm.weight", H),
                                  **{k: C.cast(v, C.POINTER(_capi.IgTensor)) for k, v in per.items()})
        c = cfg.to_c()
        h = C.c_void_p()
        if isinstance(device, (list, tuple)):
            devs = (C.c_int32 * len(device))(*device)
            _capi.check(lib.ig_model_create_stored_multi(C.byref(c), C.byref(w), devs, len(device), C.byref(h)))
        else:
            _capi.check(lib.ig_model_create_stored(C.byref(c), C.byref(w), device, C.byref(h)))
        m = cls(cfg, h, device)
        m.SetEmbeddingTable(table)
        return m

    def replica(self, i: int):
        """(handle, device) of replica i: the handle that the device-buffer
        entry points take for that GPU (borrowed; it lives with the model)."""
        h, d = C.c_void_p(), C.c_int32()
        _capi.check(_capi.load().ig_model_replica(self._h, i, C.byref(h), C.byref(d)))
        return h, d.value

    def device_count(self) -> int:
        n = C.c_int32()
        _capi.check(_capi.load().ig_model_device_count(self._h, C.byref(n)))
        return n.value

    def close(self):
        if getattr(self, "_h", None):
            _capi.load().ig_model_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- embedding table (infer.go:12-25, embeddings.go) ----
    def SetEmbeddingTable(self, t: "MappedEmbeddings"):
        """Replaces the float32 table with t, uploaded in its stored format and
        widened in the embedding gather."""
        if t.i8 is not None:
            tab = _capi.IgEmbeddingTable(format=_capi.IG_EMB_INT8, i8=t.i8.ctypes.data, scale=t.scale.ctypes.data)
        else:
            tab = _capi.IgEmbeddingTable(format=_capi.IG_EMB_BF16, bf16=t.bf16.ctypes.data, n_exact=len(t.exact_ids),
                                         exact_ids=t.exact_ids.ctypes.data, exact_rows=t.exact_rows.ctypes.data)
        _capi.check(_capi.load().ig_model_set_embeddings(self._h, C.byref(tab)))
        self.emb_table = t

    # ---- switches (infer.go:115-135) ----
    def SetInt8(self, on: bool):
        """SetInt8 (infer.go:115-135): int8 layers (the default here), or the
        reference's float32 path on the device."""
        _capi.check(_capi.load().ig_model_set_int8(self._h, 1 if on else 0))
        self._int8 = bool(on)

    # ---- inference (infer.go:237-299) ----
    def _run(self, seqs, mode):
        ids, offs = _concat(seqs)
        nseq = len(offs) - 1
        H = self.Cfg.hidden_size
        rows = nseq if mode == _capi.IG_MODE_POOLED else int(offs[-1])
        out = np.empty((rows, H), np.float32)  # every row is written
        rc = _capi.load().ig_encode(self._h, ids.ctypes.data, offs.ctypes.data, nseq, mode, out.ctypes.data,
                                    out.size)
        if rc == _capi.IG_ERR_OUT_OF_VOCAB:
            raise ModernBertError(_capi.last_error())
        _capi.check(rc)
        return out

    def EncodeSeqs(self, seqs) -> np.ndarray:
        """Pooled embedding [B, H] of unpadded sequences (infer.go:255-289)."""
        return self._run(seqs, _capi.IG_MODE_POOLED)

    def EncodeTokens(self, seqs) -> np.ndarray:
        """Final state of every token, laid end to end [sum of lengths, H] (infer.go:291-299)."""
        return self._run(seqs, _capi.IG_MODE_TOKENS)

    def Encode(self, b: Batch) -> np.ndarray:
        """Pooled embedding of a padded batch (infer.go:237-253)."""
        if len(b.IDs) != b.B() * b.T:
            raise ModernBertError("modernbert: inconsistent batch")
        return self.EncodeSeqs([b.IDs[i * b.T:i * b.T + n] for i, n in enumerate(b.Lens)])

    def encode_dump(self, seqs, layer: int, mode=_capi.IG_MODE_POOLED):
        """EncodeSeqs plus the intermediates of one layer (parity tests)."""
        ids, offs = _concat(seqs)
        nseq = len(offs) - 1
        N = int(offs[-1])
        H, I = self.Cfg.hidden_size, self.Cfg.intermediate_size
        arr = dict(xq=np.zeros((N, H), np.uint8), xq_s=np.zeros(N, np.float32), qkv=np.zeros((N, 3 * H), np.float32),
                   ctx=np.zeros((N, H), np.float32), cq=np.zeros((N, H), np.uint8), cq_s=np.zeros(N, np.float32),
                   x_attn=np.zeros((N, H), np.float32), hq=np.zeros((N, H), np.uint8), hq_s=np.zeros(N, np.float32),
                   g=np.zeros((N, I), np.float32), gq=np.zeros((N, I), np.uint8), gq_s=np.zeros(N, np.float32),
                   x_mlp=np.zeros((N, H), np.float32), emb_ln=np.zeros((N, H), np.float32))
        d = _capi.IgDump(layer=layer, **{k: v.ctypes.data for k, v in arr.items()})
        rows = nseq if mode == _capi.IG_MODE_POOLED else N
        out = np.zeros((rows, H), np.float32)
        _capi.check(_capi.load().ig_encode_dump(self._h, ids.ctypes.data, offs.ctypes.data, nseq, mode,
                                                out.ctypes.data, out.size, C.byref(d)))
        return out, arr

    # ---- heads (heads.go) ----
    def SetHeads(self, heads: list["Head"]):
        hs = (_capi.IgHead * len(heads))()
        for i, h in enumerate(heads):
            hs[i] = _capi.IgHead(rows=h.rows, per_token=1 if h.kind == "spans" else 0, w=h.w.ctypes.data,
                                 b=h.b.ctypes.data)
        _capi.check(_capi.load().ig_model_set_heads(self._h, len(heads), hs))
        self.heads = list(heads)

    def Logits(self, seqs):
        """float64 logits of every pooled head per sequence, and of every span head per token."""
        ids, offs = _concat(seqs)
        nseq = len(offs) - 1
        N = int(offs[-1])
        pr = sum(h.rows for h in self.heads if h.kind != "spans")
        tr = sum(h.rows for h in self.heads if h.kind == "spans")
        z = np.empty((nseq, pr), np.float64)  # every entry is written
        zt = np.empty((N, tr), np.float64) if tr else None
        rc = _capi.load().ig_logits(self._h, ids.ctypes.data, offs.ctypes.data, nseq, z.ctypes.data, z.size,
                                    zt.ctypes.data if zt is not None else None, zt.size if zt is not None else 0)
        if rc == _capi.IG_ERR_OUT_OF_VOCAB:
            raise ModernBertError(_capi.last_error())
        _capi.check(rc)
        out, po, to = [], 0, 0
        for h in self.heads:
            if h.kind == "spans":
                out.append(zt[:, to:to + h.rows])
                to += h.rows
            else:
                out.append(z[:, po:po + h.rows])
                po += h.rows
        return out, offs


# ---- decision heads: answers from logits (heads.go:124-237) ----

def sigmoid(z: float) -> float:
    if z >= 0:
        return 1 / (1 + math.exp(-z))
    e = math.exp(z)
    return e / (1 + e)


def softmax(z):
    mx = max(z)
    p = [math.exp(v - mx) for v in z]
    s = 0.0
    for v in p:
        s += v
    return [v / s for v in p]


def margin(p, best):
    if len(p) < 2:
        return p[best]
    others = 0.0
    for i, v in enumerate(p):
        if i != best:
            others += v
    return p[best] - others / (len(p) - 1)


@dataclass
class Head:
    """A question's output layer (heads.go:19-27)."""
    name: str
    kind: str  # noul | choice | score | spans
    w: np.ndarray
    b: np.ndarray
    options: list = field(default_factory=list)

    @property
    def rows(self) -> int:
        return self.w.shape[0]

    def answer(self, z, temperature: float = 1.0) -> dict:
        """head.answer (heads.go:124-187)."""
        if temperature <= 0:
            temperature = 1
        zt = [float(v) / temperature for v in z]
        a = dict(question=self.name, kind=self.kind)
        opts = self.options or [str(i) for i in range(len(zt) + (1 if self.kind == "score" else 0))]
        if self.kind == "noul":
            a["P"] = sigmoid(zt[0])
            a["Confidence"] = max(a["P"], 1 - a["P"])
        elif self.kind == "choice":
            p = softmax(zt)
            best = 0
            for i, v in enumerate(p):
                if v > p[best]:
                    best = i
            a["Probs"] = {opts[i]: v for i, v in enumerate(p)}
            a["Choice"], a["Confidence"], a["Margin"] = opts[best], p[best], margin(p, best)
        elif self.kind == "score":
            gt = []
            for k, v in enumerate(zt):
                g = sigmoid(v)
                if k > 0:
                    g = min(g, gt[k - 1])
                gt.append(g)
            levels = len(opts)
            dist = []
            for k in range(levels):
                above = 1.0 if k == 0 else gt[k - 1]
                below = gt[k] if k < len(gt) else 0.0
                dist.append(above - below)
            best, score = 0, 0.0
            for k, v in enumerate(dist):
                score += k * v
                if v > dist[best]:
                    best = k
            a["Probs"] = {opts[k]: v for k, v in enumerate(dist)}
            a["Score"], a["Choice"], a["Confidence"] = score, opts[best], dist[best]
        return a
