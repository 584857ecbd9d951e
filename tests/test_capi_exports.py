"""The C-ABI library builds, loads without a GPU and exports every symbol
include/indecis_b200.h declares (no compute calls here)."""
import ctypes
import os
import re

from indecis_b200 import _capi, build

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_header_symbols_exported():
    build.build()
    header = open(os.path.join(ROOT, "include", "indecis_b200.h")).read()
    declared = set(re.findall(r"IG_API\s+[\w\s\*]+?\b(ig_\w+)\s*\(", header))
    assert declared == set(_capi.SYMBOLS)
    lib = ctypes.CDLL(_capi.LIB_PATH)
    for name in declared:
        assert hasattr(lib, name), name


def test_no_oracle_in_product():
    """The product path never imports or links the oracle."""
    pkg = os.path.join(ROOT, "indecis_b200")
    for dirpath, _, files in os.walk(pkg):
        for f in files:
            if f.endswith((".py", ".cu", ".cuh", ".h", ".cpp")):
                text = open(os.path.join(dirpath, f)).read()
                assert "import oracle" not in text and "liboracle" not in text and "or_encode" not in text, f


def test_errors_without_device():
    """Creating a model with no usable device fails with a status, not a crash."""
    _capi.load()
    import numpy as np
    from indecis_b200 import synthetic as S
    from indecis_b200.model import Config, Model
    import torch
    if torch.cuda.is_available():
        return
    cfg = S.tiny(layers=1, hidden=128, heads=2, intermediate=128, vocab=64)
    W = S.weights(cfg)
    try:
        Model.from_arrays(Config.from_dict(cfg), W)
    except _capi.IgError as e:
        assert e.code == _capi.IG_ERR_NO_DEVICE
    else:
        raise AssertionError("expected IG_ERR_NO_DEVICE")
