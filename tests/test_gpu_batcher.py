"""The batching front end on the device: concurrent callers' requests go
through one queue into batches on two models (two GPUs' worth of workers,
here on one device), and each caller gets EncodeSeqs' bits for its own
sequences (batch composition does not change a sequence's result:
concurrency_test.go:12)."""
import threading

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_batcher_bitexact(igdev):
    from indecis_b200 import synthetic as S
    from indecis_b200.batch import Batcher
    from indecis_b200.model import Config, ModernBertError, Model
    cfg = S.tiny(layers=3, hidden=128, heads=2, intermediate=192, vocab=900)
    W = S.weights(cfg, seed=17)
    models = [Model.from_arrays(Config.from_dict(cfg), W) for _ in range(2)]
    ref = models[0]
    b = Batcher(models, workers=2, max_rows=2048, max_wait_us=2000)
    rng = np.random.default_rng(5)
    reqs = [[rng.integers(0, 900, int(rng.integers(1, 200))).tolist() for _ in range(int(rng.integers(1, 5)))]
            for _ in range(160)]
    reqs[7] = [[3, 4, 900]]  # out of vocabulary: fails alone
    res, errs = [None] * len(reqs), [None] * len(reqs)

    def client(t):
        for i in range(t, len(reqs), 16):
            try:
                res[i] = b.encode(reqs[i])
            except ModernBertError as e:
                errs[i] = e

    ts = [threading.Thread(target=client, args=(t,)) for t in range(16)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    st = b.stats()
    b.close()
    assert "out of vocabulary" in str(errs[7])
    for i, (r, got) in enumerate(zip(reqs, res)):
        if i == 7:
            continue
        assert errs[i] is None
        assert np.array_equal(got.view(np.uint32), ref.EncodeSeqs(r).view(np.uint32))
    assert st["requests"] == 160 and st["batches"] < 160
