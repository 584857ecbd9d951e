"""The batching front end (WithBatching, model.go:137-160; batch.go): the
EncodeSeqs requests of concurrent callers coalesced into device batches by
the library's C++ workers (ig_batcher_*). One queue feeds every model given
(one per GPU); `max_wait_us` lets a worker wait for more requests while its
batch is short (0: the reference's behaviour, never wait).
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _capi


class Batcher:
    """Thread-safe: call encode() from as many threads as there are clients."""

    def __init__(self, models=None, workers: int = 2, max_rows: int = 512, max_wait_us: int = 0, *, encode_fn=None,
                 hidden: int = 0, devices: int = 1):
        L = _capi.load()
        h = C.c_void_p()
        self._cb = None
        if encode_fn is not None:
            # Any encoder: encode_fn(device, ids, offs) -> pooled [nseq][hidden] (or raises).
            def cb(user, ids, offs, nseq, out):
                try:
                    o = np.ctypeslib.as_array(offs, shape=(nseq + 1,)).copy()
                    i = np.ctypeslib.as_array(ids, shape=(max(int(o[-1]), 1),))[:int(o[-1])].copy()
                    res = np.ascontiguousarray(encode_fn(int(user or 0), i, o), np.float32)
                    C.memmove(out, res.ctypes.data, res.nbytes)
                    return 0
                except Exception:
                    return _capi.IG_ERR_OUT_OF_VOCAB

            self._cb = _capi.BATCH_ENCODE_FN(cb)
            users = (C.c_void_p * devices)(*range(devices))
            rc = L.ig_batcher_create_fn(self._cb, users, devices, hidden, workers, max_rows, max_wait_us, C.byref(h))
            self.hidden = hidden
        else:
            models = list(models)
            arr = (C.c_void_p * len(models))(*[m._h for m in models])
            rc = L.ig_batcher_create(arr, len(models), workers, max_rows, max_wait_us, C.byref(h))
            self.hidden = models[0].Cfg.hidden_size
            self._models = models  # kept alive while the workers use them
        _capi.check(rc)
        self._h = h.value

    def encode(self, seqs) -> np.ndarray:
        """EncodeSeqs through the batcher: pooled [nseq][hidden]."""
        from .model import ModernBertError, _concat
        ids, offs = _concat(seqs)
        nseq = len(offs) - 1
        out = np.zeros((nseq, self.hidden), np.float32)
        rc = _capi.load().ig_batcher_encode(self._h, ids.ctypes.data, offs.ctypes.data, nseq, out.ctypes.data, out.size)
        if rc == _capi.IG_ERR_OUT_OF_VOCAB:
            raise ModernBertError(_capi.last_error())
        _capi.check(rc)
        return out

    def stats(self) -> dict:
        r, b, n = C.c_int64(), C.c_int64(), C.c_int64()
        _capi.load().ig_batcher_stats(self._h, C.byref(r), C.byref(b), C.byref(n))
        return dict(requests=r.value, batches=b.value, rows=n.value)

    def close(self):
        if getattr(self, "_h", None):
            _capi.load().ig_batcher_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
