"""ctypes binding of libindecis_b200.so (include/indecis_b200.h).

Loading fails loudly when the library has not been built: there is no
fallback implementation of any entry point.
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libindecis_b200.so")

IG_OK = 0
IG_ERR_BAD_ARG = 1
IG_ERR_OUT_OF_VOCAB = 2
IG_ERR_CUDA = 3
IG_ERR_TIMEOUT = 4
IG_ERR_UNSUPPORTED = 5
IG_ERR_NO_DEVICE = 6
IG_MODE_POOLED = 0
IG_MODE_TOKENS = 1

# Every symbol the header declares (tests check the library exports them all).
SYMBOLS = ["ig_model_create", "ig_model_destroy", "ig_model_set_heads", "ig_encode", "ig_encode_device",
           "ig_logits", "ig_last_error", "ig_device_error", "ig_gemm_u8s8", "ig_quantize_rows",
           "ig_layernorm_quant", "ig_pack_b8", "ig_attention", "ig_encode_dump", "ig_logits_device",
           "ig_profile", "ig_profile_report", "ig_attention_noalloc", "ig_model_set_embeddings",
           "ig_plan_windows", "ig_log_softmax", "ig_decode_spans", "ig_answer_spans", "ig_window_logits",
           "ig_infer_windows", "ig_model_head_rows", "ig_vision_create", "ig_vision_destroy", "ig_vision_forward",
           "ig_vision_forward_device", "ig_vision_dump_layer", "ig_model_dims", "ig_batcher_create",
           "ig_batcher_create_fn", "ig_batcher_destroy", "ig_batcher_encode", "ig_batcher_stats",
           "ig_spans_tags_device", "ig_spans_tags", "ig_spans_from_tags", "ig_model_set_int8",
           "ig_check_gelu_division", "ig_model_create_multi", "ig_model_replica", "ig_model_device_count",
           "ig_model_create_stored", "ig_model_create_stored_multi", "ig_device_count", "ig_gemm_geglu_quant",
           "ig_profile_only", "ig_check_wait_timeout"]

IG_EMB_F32 = 0
IG_EMB_BF16 = 1
IG_EMB_INT8 = 2


class IgConfig(C.Structure):
    _fields_ = [("vocab", C.c_int32), ("hidden", C.c_int32), ("layers", C.c_int32), ("heads", C.c_int32),
                ("intermediate", C.c_int32), ("global_every", C.c_int32), ("local_attention", C.c_int32),
                ("pooling", C.c_int32), ("norm_eps", C.c_double), ("global_theta", C.c_double),
                ("local_theta", C.c_double), ("simd_lanes", C.c_int32)]


class IgWeights(C.Structure):
    _fields_ = [("tok_embeddings", C.c_void_p), ("emb_norm", C.c_void_p), ("final_norm", C.c_void_p),
                ("attn_norm", C.POINTER(C.c_void_p)), ("wqkv", C.POINTER(C.c_void_p)),
                ("wo", C.POINTER(C.c_void_p)), ("mlp_norm", C.POINTER(C.c_void_p)),
                ("wi", C.POINTER(C.c_void_p)), ("wo_mlp", C.POINTER(C.c_void_p))]


IG_DT = {"F32": 0, "BF16": 1, "F16": 2, "I8": 3}


class IgTensor(C.Structure):
    _fields_ = [("dtype", C.c_int32), ("data", C.c_void_p)]


class IgStoredWeights(C.Structure):
    _fields_ = [("emb_norm", IgTensor), ("final_norm", IgTensor), ("attn_norm", C.POINTER(IgTensor)),
                ("wqkv", C.POINTER(IgTensor)), ("wo", C.POINTER(IgTensor)), ("mlp_norm", C.POINTER(IgTensor)),
                ("wi", C.POINTER(IgTensor)), ("wo_mlp", C.POINTER(IgTensor))]


class IgEmbeddingTable(C.Structure):
    _fields_ = [("format", C.c_int32), ("f32", C.c_void_p), ("bf16", C.c_void_p), ("n_exact", C.c_int32),
                ("exact_ids", C.c_void_p), ("exact_rows", C.c_void_p), ("i8", C.c_void_p), ("scale", C.c_void_p)]


class IgHead(C.Structure):
    _fields_ = [("rows", C.c_int32), ("per_token", C.c_int32), ("w", C.c_void_p), ("b", C.c_void_p)]


class IgWindow(C.Structure):
    _fields_ = [("start", C.c_int32), ("end", C.c_int32), ("keep_from", C.c_int32), ("keep_to", C.c_int32)]


class IgSpan(C.Structure):
    _fields_ = [("type", C.c_int32), ("start", C.c_int32), ("end", C.c_int32), ("confidence", C.c_double)]


BATCH_ENCODE_FN = C.CFUNCTYPE(C.c_int, C.c_void_p, C.POINTER(C.c_int32), C.POINTER(C.c_int64), C.c_int32,
                             C.POINTER(C.c_float))


class IgVisionConfig(C.Structure):
    _fields_ = [("hidden", C.c_int32), ("layers", C.c_int32), ("heads", C.c_int32), ("mlp", C.c_int32),
                ("image_size", C.c_int32), ("patch_size", C.c_int32), ("eps", C.c_double), ("simd_lanes", C.c_int32)]


VISION_FLAT = ("patch_w", "patch_b", "pos")
VISION_LAYER = ("ln1_g", "ln1_b", "ln2_g", "ln2_b", "wqkv", "bqkv", "wo", "bo", "w1", "b1", "w2", "b2")
VISION_TAIL = ("post_g", "post_b", "probe", "in_w", "in_b", "hout_w", "hout_b", "hln_g", "hln_b", "hfc1_w", "hfc1_b",
               "hfc2_w", "hfc2_b")


class IgVisionWeights(C.Structure):
    _fields_ = ([(n, C.c_void_p) for n in VISION_FLAT] + [(n, C.POINTER(C.c_void_p)) for n in VISION_LAYER] +
                [(n, C.c_void_p) for n in VISION_TAIL])


class IgVisionDump(C.Structure):
    _fields_ = [("layer", C.c_int32)] + [(n, C.c_void_p) for n in (
        "x_embed", "h1q", "h1q_s", "qkv", "attn", "x_attn", "h2q", "h2q_s", "mlp", "outliers", "noutliers", "mq",
        "mq_s", "x_mlp")]


class IgDump(C.Structure):
    _fields_ = [("layer", C.c_int32)] + [(n, C.c_void_p) for n in (
        "xq", "xq_s", "qkv", "ctx", "cq", "cq_s", "x_attn", "hq", "hq_s", "g", "gq", "gq_s", "x_mlp", "emb_ln")]


_lib = None


class LibraryMissing(RuntimeError):
    pass


def load() -> C.CDLL:
    """Loads the in-tree library (built by indecis_b200.build)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise LibraryMissing(f"{LIB_PATH} is not built: run `python -m indecis_b200.build` (no CPU fallback exists)")
    L = C.CDLL(LIB_PATH)
    vp, i32, i64p = C.c_void_p, C.c_int32, C.POINTER(C.c_int64)
    i32p = C.POINTER(C.c_int32)
    L.ig_model_create.argtypes = [C.POINTER(IgConfig), C.POINTER(IgWeights), i32, C.POINTER(C.c_void_p)]
    L.ig_model_create.restype = C.c_int
    L.ig_model_create_multi.argtypes = [C.POINTER(IgConfig), C.POINTER(IgWeights), i32p, i32, C.POINTER(C.c_void_p)]
    L.ig_model_create_stored.argtypes = [C.POINTER(IgConfig), C.POINTER(IgStoredWeights), i32, C.POINTER(C.c_void_p)]
    L.ig_model_create_stored_multi.argtypes = [C.POINTER(IgConfig), C.POINTER(IgStoredWeights), i32p, i32,
                                               C.POINTER(C.c_void_p)]
    L.ig_model_replica.argtypes = [vp, i32, C.POINTER(C.c_void_p), i32p]
    L.ig_model_device_count.argtypes = [vp, i32p]
    L.ig_device_count.argtypes = [i32p]
    L.ig_model_destroy.argtypes = [vp]
    L.ig_model_destroy.restype = None
    L.ig_model_set_heads.argtypes = [vp, i32, C.POINTER(IgHead)]
    L.ig_encode.argtypes = [vp, vp, vp, i32, i32, vp, C.c_size_t]
    L.ig_encode_device.argtypes = [vp, vp, vp, i32, i32, vp, vp]
    L.ig_logits.argtypes = [vp, vp, vp, i32, vp, C.c_size_t, vp, C.c_size_t]
    L.ig_last_error.restype = C.c_char_p
    L.ig_device_error.argtypes = [i32]
    L.ig_device_error.restype = i32
    L.ig_gemm_u8s8.argtypes = [vp, i32, vp, i32, i32, i32, i32, vp, vp, vp, vp, i32, i32, vp, vp]
    L.ig_quantize_rows.argtypes = [vp, i32, i32, i32, vp, i32, vp, vp]
    L.ig_gemm_geglu_quant.argtypes = [vp, i32, vp, i32, i32, i32, i32, vp, vp, vp, vp, i32, vp, vp]
    L.ig_layernorm_quant.argtypes = [vp, vp, i32, i32, C.c_double, i32, vp, vp, i32, vp, vp]
    L.ig_pack_b8.argtypes = [vp, i32, i32, vp, i32, vp, vp, vp, vp]
    L.ig_attention.argtypes = [vp, i32, i32, vp, i32, i32, i32, vp, vp]
    L.ig_encode_dump.argtypes = [vp, vp, vp, i32, i32, vp, C.c_size_t, C.POINTER(IgDump)]
    L.ig_logits_device.argtypes = [vp, vp, vp, i32, vp, vp, vp]
    L.ig_attention_noalloc.argtypes = [vp, i32, i32, vp, i32, i32, i32, vp, vp]
    L.ig_check_gelu_division.argtypes = [vp, vp, vp]
    L.ig_check_wait_timeout.argtypes = [C.c_int64, vp, vp]
    L.ig_model_set_embeddings.argtypes = [vp, C.POINTER(IgEmbeddingTable)]
    f64 = C.c_double
    L.ig_plan_windows.argtypes = [i32, i32, i32, C.POINTER(IgWindow), i32, i32p]
    L.ig_log_softmax.argtypes = [vp, i32, f64, vp]
    L.ig_decode_spans.argtypes = [vp, i32, i32, f64, C.c_char_p, C.c_int64, vp, vp, C.POINTER(IgSpan), i32, i32p]
    L.ig_answer_spans.argtypes = [vp, i32, i32, i32, f64, f64, C.c_char_p, C.c_int64, vp, C.POINTER(IgSpan), i32,
                                  i32p]
    L.ig_window_logits.argtypes = [vp, vp, vp, i32, vp, C.c_size_t, vp, C.c_size_t]
    L.ig_infer_windows.argtypes = [vp, vp, vp, i32, vp, i32, vp, i32, i32, i32, vp, C.c_size_t, vp, C.c_size_t]
    L.ig_model_head_rows.argtypes = [vp, i32p, i32p]
    L.ig_vision_create.argtypes = [C.POINTER(IgVisionConfig), C.POINTER(IgVisionWeights), i32, C.POINTER(C.c_void_p)]
    L.ig_vision_destroy.argtypes = [vp]
    L.ig_vision_destroy.restype = None
    L.ig_vision_forward.argtypes = [vp, vp, i32, i32, vp, C.c_size_t, vp, C.c_size_t]
    L.ig_vision_forward_device.argtypes = [vp, vp, i32, i32, vp, vp, vp]
    L.ig_vision_dump_layer.argtypes = [vp, vp, i32, C.POINTER(IgVisionDump), vp, C.c_size_t]
    L.ig_model_dims.argtypes = [vp, i32p, i32p]
    L.ig_model_set_int8.argtypes = [vp, i32]
    L.ig_spans_tags_device.argtypes = [vp, C.c_int64, vp, i32, i32, f64, f64, vp, vp]
    L.ig_spans_tags.argtypes = [vp, C.c_int64, vp, i32, i32, f64, f64, vp, i32]
    L.ig_spans_from_tags.argtypes = [vp, i32, i32, i32, f64, vp, C.c_char_p, C.c_int64, vp, C.POINTER(IgSpan), i32,
                                     i32p]
    L.ig_batcher_create.argtypes = [C.POINTER(C.c_void_p), i32, i32, i32, i32, C.POINTER(C.c_void_p)]
    L.ig_batcher_create_fn.argtypes = [BATCH_ENCODE_FN, C.POINTER(C.c_void_p), i32, i32, i32, i32, i32,
                                       C.POINTER(C.c_void_p)]
    L.ig_batcher_destroy.argtypes = [vp]
    L.ig_batcher_destroy.restype = None
    L.ig_batcher_encode.argtypes = [vp, vp, vp, i32, vp, C.c_size_t]
    L.ig_batcher_stats.argtypes = [vp, C.POINTER(C.c_int64), C.POINTER(C.c_int64), C.POINTER(C.c_int64)]
    L.ig_profile.argtypes = [i32]
    L.ig_profile_only.argtypes = [C.c_char_p]
    L.ig_profile_report.argtypes = [C.c_char_p, C.c_size_t]
    L.ig_profile_report.restype = C.c_int64
    _lib = L
    return L


def last_error() -> str:
    return load().ig_last_error().decode()


class IgError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(msg or f"indecis_b200 error {code}")
        self.code = code


def profile(enable: bool):
    check(load().ig_profile(1 if enable else 0))


def profile_only(name: str | None):
    """Events around the launches recorded under `name` only (None: every launch)."""
    check(load().ig_profile_only(name.encode() if name else None))


def profile_report() -> dict:
    """Per-kernel totals since profile(True) (synchronizes the device)."""
    import json
    L = load()
    n = L.ig_profile_report(None, 0)
    buf = C.create_string_buffer(int(n) + 1)
    L.ig_profile_report(buf, len(buf))
    return json.loads(buf.value.decode())


def check(rc: int):
    if rc != IG_OK:
        raise IgError(rc, last_error())
