"""CPU oracle for the int8 ModernBERT encoder path (TEST INFRASTRUCTURE).

This package is the checker the CUDA path is compared against and the CPU
baseline that ``bench.py`` times. Only ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py``'s CPU legs may import it; the product (``indecis_b200``) never
does. See ``oracle/oracle.h`` for the restated reference functions, their
file:line citations and the parity status ("parity unpinned" for the composite
encoder: the Go reference cannot run here and ships no int8 golden vectors;
the elementary operations are pinned by the reference's own known-answer and
property tests).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = os.path.join(_HERE, "liboracle.so")
_lib = None

f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
f64p = np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")
i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
i64p = np.ctypeslib.ndpointer(np.int64, flags="C_CONTIGUOUS")
u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
i8p = np.ctypeslib.ndpointer(np.int8, flags="C_CONTIGUOUS")


def build() -> str:
    """Compile liboracle.so with the committed Makefile (g++, no CUDA)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB


class Config(C.Structure):
    _fields_ = [("vocab", C.c_int), ("hidden", C.c_int), ("layers", C.c_int), ("heads", C.c_int),
                ("intermediate", C.c_int), ("global_every", C.c_int), ("local_attention", C.c_int),
                ("cls", C.c_int), ("norm_eps", C.c_double), ("global_theta", C.c_double),
                ("local_theta", C.c_double), ("V", C.c_int)]


class Weights(C.Structure):
    _fields_ = [("emb", C.c_void_p), ("emb_norm", C.c_void_p), ("final_norm", C.c_void_p),
                ("attn_norm", C.POINTER(C.c_void_p)), ("wqkv", C.POINTER(C.c_void_p)),
                ("wo", C.POINTER(C.c_void_p)), ("mlp_norm", C.POINTER(C.c_void_p)),
                ("wi", C.POINTER(C.c_void_p)), ("wo_mlp", C.POINTER(C.c_void_p))]


_DUMP_FIELDS = [("layer", C.c_int), ("xq", C.c_void_p), ("xq_s", C.c_void_p), ("qkv_acc", C.c_void_p),
                ("qkv", C.c_void_p), ("ctx", C.c_void_p), ("cq", C.c_void_p), ("cq_s", C.c_void_p),
                ("x_attn", C.c_void_p), ("hq", C.c_void_p), ("hq_s", C.c_void_p), ("z", C.c_void_p),
                ("gq", C.c_void_p), ("gq_s", C.c_void_p), ("x_mlp", C.c_void_p), ("emb_ln", C.c_void_p)]


class Dump(C.Structure):
    _fields_ = _DUMP_FIELDS


class AttnDbg(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in ("qa", "sq", "kq", "ks", "kzc", "vq", "vs", "kmean", "p", "sp",
                                          "sacc", "oacc")]


def lib():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(_LIB):
        build()
    L = C.CDLL(_LIB)
    L.or_round_half_even.restype = C.c_float
    L.or_round_half_even.argtypes = [C.c_float]
    L.or_exp32.restype = C.c_float
    L.or_exp32.argtypes = [C.c_float]
    L.or_erf32.restype = C.c_float
    L.or_erf32.argtypes = [C.c_float]
    L.or_exp_shift.restype = C.c_float
    L.or_exp_shift.argtypes = [f32p, C.c_int, C.c_float, C.c_int]
    L.or_gelu_mul.argtypes = [f32p, f32p, f32p, C.c_int]
    L.or_layernorm_row.argtypes = [f32p, f32p, f32p, C.c_int, C.c_double, C.c_int]
    L.or_rope.argtypes = [f32p, f32p, f32p, C.c_int]
    L.or_rope_table.argtypes = [C.c_double, C.c_int, C.c_int, f32p, f32p]
    L.or_quant_row.restype = C.c_float
    L.or_quant_row.argtypes = [i8p, f32p, C.c_void_p, C.c_int, C.c_int, C.POINTER(C.c_int32)]
    L.or_pack_b8.argtypes = [f32p, C.c_int, C.c_int, C.c_int, i8p, f32p, i32p, f32p]
    L.or_quantize_a.argtypes = [f32p, C.c_int, C.c_int, u8p, f32p]
    L.or_gemm_u8s8.argtypes = [u8p, C.c_int, i8p, C.c_int, C.c_int, C.c_int, C.c_int, i32p]
    L.or_dequant.argtypes = [i32p, C.c_int, C.c_int, f32p, f32p, f32p, f32p, C.c_int]
    L.or_matmul8.argtypes = [f32p, f32p, C.c_int, i8p, f32p, f32p, C.c_int, C.c_int, C.c_int]
    L.or_attn8.argtypes = [f32p, f32p, f32p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float, f32p, C.c_int,
                           C.c_void_p]
    L.or_model_create.restype = C.c_void_p
    L.or_model_create.argtypes = [C.POINTER(Config), C.POINTER(Weights)]
    L.or_model_destroy.argtypes = [C.c_void_p]
    L.or_encode.restype = C.c_int
    L.or_encode.argtypes = [C.c_void_p, i32p, i64p, C.c_int, C.c_int, f32p, C.c_int, C.c_int, C.c_void_p,
                            C.POINTER(C.c_int32)]
    L.or_head_logits.argtypes = [f32p, f32p, C.c_int, C.c_int, f32p, C.c_int, f64p]
    L.or_encode_f32.restype = C.c_int
    L.or_encode_f32.argtypes = [C.c_void_p, i32p, i64p, C.c_int, C.c_int, f32p, C.c_int, C.POINTER(C.c_int32)]
    L.or_cpu_features.restype = C.c_int
    L.or_phase_seconds.argtypes = [f64p, C.c_int]
    L.or_siglip_create.restype = C.c_void_p
    L.or_siglip_create.argtypes = [C.c_void_p, C.c_void_p]
    L.or_siglip_destroy.argtypes = [C.c_void_p]
    L.or_siglip_forward.restype = C.c_int
    L.or_siglip_forward.argtypes = [C.c_void_p, f32p, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_int, C.c_int,
                                    C.c_void_p]
    L.or_linear_f32.argtypes = [f32p, f32p, C.c_int, f32p, C.c_void_p, C.c_int, C.c_int]
    L.or_gelu_tanh.argtypes = [f32p, f32p, C.c_int, C.c_int]
    L.or_siglip_softmax.argtypes = [f32p, C.c_int, C.c_float, C.c_int]
    L.or_matmul8_outliers.argtypes = [f32p, f32p, C.c_int, i8p, f32p, f32p, C.c_int, C.c_int, C.c_float, i32p,
                                      C.POINTER(C.c_int32)]
    _lib = L
    return L


# ---- thin numpy wrappers ----------------------------------------------------


def phase_seconds(reset: bool = True):
    """Wall seconds of the encoder's phases since the last reset:
    (norms + QKV + RoPE, attention, output projection + norm + MLP)."""
    out = np.zeros(3, np.float64)
    lib().or_phase_seconds(out, 1 if reset else 0)
    return tuple(float(v) for v in out)

def round_half_even(v: float) -> float:
    return lib().or_round_half_even(v)


def exp_shift(x, m, V=8):
    x = np.ascontiguousarray(x, np.float32).copy()
    s = lib().or_exp_shift(x, x.size, m, V)
    return x, s


def gelu_mul(a, b):
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    o = np.empty_like(a)
    lib().or_gelu_mul(o, a, b, a.size)
    return o


def layernorm(x, gamma, eps=1e-5, V=8):
    x = np.ascontiguousarray(x, np.float32)
    o = np.empty_like(x)
    g = np.ascontiguousarray(gamma, np.float32)
    for r in range(x.shape[0]):
        lib().or_layernorm_row(o[r], x[r], g, x.shape[1], eps, V)
    return o


def rope_table(theta, D, npos):
    c = np.empty((npos, D // 2), np.float32)
    s = np.empty((npos, D // 2), np.float32)
    lib().or_rope_table(theta, D, npos, c, s)
    return c, s


def pack_b8(w, transB=True):
    """w: [n, k] (transB) float32 -> (q int8 [n, k], scale [n], colsum [n], zc [n])."""
    w = np.ascontiguousarray(w, np.float32)
    n, k = w.shape if transB else (w.shape[1], w.shape[0])
    q = np.empty((n, k), np.int8)
    s = np.empty(n, np.float32)
    cs = np.empty(n, np.int32)
    zc = np.empty(n, np.float32)
    lib().or_pack_b8(w, k, n, 1 if transB else 0, q, s, cs, zc)
    return q, s, cs, zc


def quantize_a(a):
    a = np.ascontiguousarray(a, np.float32)
    m, k = a.shape
    q = np.empty((m, k), np.uint8)
    sa = np.empty(m, np.float32)
    lib().or_quantize_a(a, m, k, q, sa)
    return q, sa


def gemm_u8s8(A, B):
    A = np.ascontiguousarray(A, np.uint8)
    B = np.ascontiguousarray(B, np.int8)
    M, K = A.shape
    N = B.shape[0]
    acc = np.empty((M, N), np.int32)
    lib().or_gemm_u8s8(A, K, B, K, M, N, K, acc)
    return acc


def dequant(acc, sa, sb, zc, C_old=None):
    acc = np.ascontiguousarray(acc, np.int32)
    M, N = acc.shape
    C = np.zeros((M, N), np.float32) if C_old is None else np.ascontiguousarray(C_old, np.float32).copy()
    lib().or_dequant(acc, M, N, np.ascontiguousarray(sa, np.float32), np.ascontiguousarray(sb, np.float32),
                     np.ascontiguousarray(zc, np.float32), C, 0 if C_old is None else 1)
    return C


def matmul8(a, q, scale, zc, c_old=None):
    a = np.ascontiguousarray(a, np.float32)
    m, k = a.shape
    n = q.shape[0]
    c = np.zeros((m, n), np.float32) if c_old is None else np.ascontiguousarray(c_old, np.float32).copy()
    lib().or_matmul8(c, a, m, np.ascontiguousarray(q), scale, zc, k, n, 0 if c_old is None else 1)
    return c


def attn8(q, k, v, window, scale, debug=False):
    """q, k, v: [n, D] float32. Returns o [n, D] (and the internals if debug)."""
    q = np.ascontiguousarray(q, np.float32)
    k = np.ascontiguousarray(k, np.float32)
    v = np.ascontiguousarray(v, np.float32)
    n, D = q.shape
    o = np.full((n, D), np.nan, np.float32)
    dbg = None
    arrays = {}
    if debug:
        arrays = dict(qa=np.zeros((n, D), np.uint8), sq=np.zeros(n, np.float32), kq=np.zeros((n, D), np.int8),
                      ks=np.zeros(n, np.float32), kzc=np.zeros(n, np.float32), vq=np.zeros((n, D), np.int8),
                      vs=np.zeros(D, np.float32), kmean=np.zeros(D, np.float32), p=np.zeros((n, n), np.uint8),
                      sp=np.zeros(n, np.float32), sacc=np.zeros((n, n), np.int32), oacc=np.zeros((n, D), np.int32))
        dbg = AttnDbg(**{kk: vv.ctypes.data for kk, vv in arrays.items()})
    if n:
        lib().or_attn8(q, k, v, D, n, D, window, scale, o, D, C.byref(dbg) if dbg is not None else None)
    return (o, arrays) if debug else o


def head_logits(w, b, x):
    w = np.ascontiguousarray(w, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    x = np.ascontiguousarray(np.atleast_2d(x), np.float32)
    rows, H = w.shape
    z = np.empty((x.shape[0], rows), np.float64)
    lib().or_head_logits(w, b, rows, H, x, x.shape[0], z)
    return z


class Model:
    """Oracle encoder over float32 weights in transformers layouts."""

    def __init__(self, cfg: dict, weights: dict):
        self.cfg = cfg
        L = cfg["layers"]
        self._keep = {k: (np.ascontiguousarray(v, np.float32) if not isinstance(v, list)
                          else [None if a is None else np.ascontiguousarray(a, np.float32) for a in v])
                      for k, v in weights.items()}
        W = self._keep

        def arr(name):
            ptrs = (C.c_void_p * L)(*[0 if a is None else a.ctypes.data for a in W[name]])
            return C.cast(ptrs, C.POINTER(C.c_void_p)), ptrs

        self._ptrs = {}
        fields = {}
        for name in ("attn_norm", "wqkv", "wo", "mlp_norm", "wi", "wo_mlp"):
            p, keep = arr(name)
            fields[name] = p
            self._ptrs[name] = keep
        w = Weights(emb=W["emb"].ctypes.data, emb_norm=W["emb_norm"].ctypes.data,
                    final_norm=W["final_norm"].ctypes.data, **fields)
        c = Config(vocab=cfg["vocab"], hidden=cfg["hidden"], layers=L, heads=cfg["heads"],
                   intermediate=cfg["intermediate"], global_every=cfg["global_every"],
                   local_attention=cfg["local_attention"], cls=1 if cfg.get("pooling") == "cls" else 0,
                   norm_eps=cfg["norm_eps"], global_theta=cfg["global_theta"], local_theta=cfg["local_theta"],
                   V=cfg.get("V", 8))
        self._h = lib().or_model_create(C.byref(c), C.byref(w))

    def __del__(self):
        if getattr(self, "_h", None):
            lib().or_model_destroy(self._h)
            self._h = None

    def encode_f32(self, ids, offs, mode=0, threads=1):
        """The float32 path (the reference without SetInt8)."""
        ids = np.ascontiguousarray(ids, np.int32)
        offs = np.ascontiguousarray(offs, np.int64)
        nseq = len(offs) - 1
        N = int(offs[-1])
        out = np.zeros((nseq if mode == 0 else N, self.cfg["hidden"]), np.float32)
        bad = C.c_int32(0)
        rc = lib().or_encode_f32(self._h, ids, offs, nseq, mode, out, threads, C.byref(bad))
        if rc == 2:
            raise ValueError("modernbert: inconsistent batch")
        if rc != 0:
            raise ValueError(f"modernbert: id {bad.value} out of vocabulary")
        return out

    def encode(self, ids, offs, mode=0, threads=1, fast=False, dump_layer=None):
        ids = np.ascontiguousarray(ids, np.int32)
        offs = np.ascontiguousarray(offs, np.int64)
        nseq = len(offs) - 1
        H = self.cfg["hidden"]
        I = self.cfg["intermediate"]
        N = int(offs[-1])
        out = np.zeros((nseq if mode == 0 else N, H), np.float32)
        dump = None
        arrays = {}
        if dump_layer is not None:
            arrays = dict(xq=np.zeros((N, H), np.uint8), xq_s=np.zeros(N, np.float32),
                          qkv_acc=np.zeros((N, 3 * H), np.int32), qkv=np.zeros((N, 3 * H), np.float32),
                          ctx=np.zeros((N, H), np.float32), cq=np.zeros((N, H), np.uint8),
                          cq_s=np.zeros(N, np.float32), x_attn=np.zeros((N, H), np.float32),
                          hq=np.zeros((N, H), np.uint8), hq_s=np.zeros(N, np.float32),
                          z=np.zeros((N, 2 * I), np.float32), gq=np.zeros((N, I), np.uint8),
                          gq_s=np.zeros(N, np.float32), x_mlp=np.zeros((N, H), np.float32),
                          emb_ln=np.zeros((N, H), np.float32))
            dump = Dump(layer=dump_layer, **{k: v.ctypes.data for k, v in arrays.items()})
        bad = C.c_int32(0)
        rc = lib().or_encode(self._h, ids, offs, nseq, mode, out, threads, 1 if fast else 0,
                             C.byref(dump) if dump is not None else None, C.byref(bad))
        if rc == 2:
            raise ValueError("modernbert: inconsistent batch")
        if rc != 0:
            raise ValueError(f"modernbert: id {bad.value} out of vocabulary")
        return (out, arrays) if dump_layer is not None else out


# ---- SigLIP vision tower (oracle/siglip.cpp) -----------------------------------

class SiglipConfig(C.Structure):
    _fields_ = [("hidden", C.c_int), ("layers", C.c_int), ("heads", C.c_int), ("mlp", C.c_int),
                ("image_size", C.c_int), ("patch_size", C.c_int), ("eps", C.c_double), ("V", C.c_int)]


SIGLIP_FLAT = ("patch_w", "patch_b", "pos")
SIGLIP_LAYER = ("ln1_g", "ln1_b", "ln2_g", "ln2_b", "wqkv", "bqkv", "wo", "bo", "w1", "b1", "w2", "b2")
SIGLIP_TAIL = ("post_g", "post_b", "probe", "in_w", "in_b", "hout_w", "hout_b", "hln_g", "hln_b", "hfc1_w", "hfc1_b",
               "hfc2_w", "hfc2_b")


class SiglipWeights(C.Structure):
    _fields_ = ([(n, C.c_void_p) for n in SIGLIP_FLAT] + [(n, C.POINTER(C.c_void_p)) for n in SIGLIP_LAYER] +
                [(n, C.c_void_p) for n in SIGLIP_TAIL])


class SiglipDump(C.Structure):
    _fields_ = [("layer", C.c_int)] + [(n, C.c_void_p) for n in (
        "x_embed", "h1q", "h1q_s", "qkv", "attn", "x_attn", "h2q", "h2q_s", "mlp", "outliers", "noutliers", "mq",
        "mq_s", "x_mlp")]


def siglip_dump_arrays(n, T, H, M):
    N = n * T
    return dict(x_embed=np.zeros((N, H), np.float32), h1q=np.zeros((N, H), np.uint8), h1q_s=np.zeros(N, np.float32),
                qkv=np.zeros((N, 3 * H), np.float32), attn=np.zeros((N, H), np.float32),
                x_attn=np.zeros((N, H), np.float32), h2q=np.zeros((N, H), np.uint8), h2q_s=np.zeros(N, np.float32),
                mlp=np.zeros((N, M), np.float32), outliers=np.zeros((n, 32), np.int32),
                noutliers=np.zeros(n, np.int32), mq=np.zeros((N, M), np.uint8), mq_s=np.zeros(N, np.float32),
                x_mlp=np.zeros((N, H), np.float32))


class SigLIP:
    """Oracle SigLIP vision tower over float32 weights (synthetic.siglip_weights layout)."""

    def __init__(self, cfg: dict, weights: dict):
        self.cfg = cfg
        L = cfg["layers"]
        self._keep = {k: (np.ascontiguousarray(v, np.float32) if not isinstance(v, list)
                          else [np.ascontiguousarray(a, np.float32) for a in v]) for k, v in weights.items()}
        W = self._keep
        self._ptrs = {}
        fields = {}
        for n in SIGLIP_FLAT + SIGLIP_TAIL:
            fields[n] = W[n].ctypes.data
        for n in SIGLIP_LAYER:
            arr = (C.c_void_p * L)(*[a.ctypes.data for a in W[n]])
            self._ptrs[n] = arr
            fields[n] = C.cast(arr, C.POINTER(C.c_void_p))
        self._w = SiglipWeights(**fields)
        self._c = SiglipConfig(hidden=cfg["hidden"], layers=L, heads=cfg["heads"], mlp=cfg["mlp"],
                               image_size=cfg["image_size"], patch_size=cfg["patch_size"], eps=cfg["eps"],
                               V=cfg.get("V", 8))
        self._h = lib().or_siglip_create(C.byref(self._c), C.byref(self._w))
        self.T = (cfg["image_size"] // cfg["patch_size"]) ** 2

    def __del__(self):
        if getattr(self, "_h", None):
            lib().or_siglip_destroy(self._h)
            self._h = None

    def forward(self, pixels, layer=0, patches=True, pooled=True, threads=1, fast=False, dump_layer=None):
        """Vision.forward on [n][3][S][S] pixels -> (patches [n][T][H] or None, pooled [n][H] or None[, dump])."""
        px = np.ascontiguousarray(pixels, np.float32)
        n, H = px.shape[0], self.cfg["hidden"]
        pa = np.zeros((n, self.T, H), np.float32) if patches else None
        po = np.zeros((n, H), np.float32) if pooled else None
        arrays, dump = {}, None
        if dump_layer is not None:
            arrays = siglip_dump_arrays(n, self.T, H, self.cfg["mlp"])
            dump = SiglipDump(layer=dump_layer, **{k: v.ctypes.data for k, v in arrays.items()})
        rc = lib().or_siglip_forward(self._h, px, n, layer, pa.ctypes.data if pa is not None else None,
                                     po.ctypes.data if po is not None else None, threads, 1 if fast else 0,
                                     C.byref(dump) if dump is not None else None)
        if rc:
            raise ValueError(f"siglip: layer {layer}, the tower has {self.cfg['layers']}")
        return (pa, po, arrays) if dump_layer is not None else (pa, po)


def linear_f32(x, W, b=None):
    x = np.ascontiguousarray(np.atleast_2d(x), np.float32)
    W = np.ascontiguousarray(W, np.float32)
    out = np.zeros((x.shape[0], W.shape[0]), np.float32)
    bb = None if b is None else np.ascontiguousarray(b, np.float32)
    lib().or_linear_f32(out, x, x.shape[0], W, bb.ctypes.data if bb is not None else None, W.shape[1], W.shape[0])
    return out


def gelu_tanh(a, V=8):
    a = np.ascontiguousarray(a, np.float32).ravel()
    o = np.zeros_like(a)
    lib().or_gelu_tanh(o, a, a.size, V)
    return o
