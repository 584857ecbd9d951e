"""The batching front end's host logic (indecis_b200/csrc/batcher.cpp) on
the CPU, with the oracle encoder standing in for the GPUs: concurrent
requests are coalesced (batch.go:54-81: the first pending request, then
those queued while the batch is under max_rows), every caller gets exactly
its rows, a failing request is answered alone, and several devices share
one queue."""
import threading

import numpy as np
import pytest

from indecis_b200 import synthetic as S
from indecis_b200.batch import Batcher


@pytest.fixture(scope="module")
def om():
    import oracle
    cfg = S.tiny(layers=2, hidden=64, heads=1, intermediate=96, vocab=300)
    return cfg, oracle.Model(cfg, S.weights(cfg, seed=4))


def _requests(n, vocab, seed):
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(n):
        k = int(rng.integers(1, 4))
        out.append([rng.integers(0, vocab, int(rng.integers(1, 30))).tolist() for _ in range(k)])
    return out


def _run_clients(b, reqs, nthreads):
    res = [None] * len(reqs)
    errs = [None] * len(reqs)

    def client(t):
        for i in range(t, len(reqs), nthreads):
            try:
                res[i] = b.encode(reqs[i])
            except Exception as e:  # noqa: BLE001
                errs[i] = e

    ts = [threading.Thread(target=client, args=(t,)) for t in range(nthreads)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    return res, errs


def test_coalesces_and_returns_each_callers_rows(om):
    cfg, model = om
    calls = []

    def enc(dev, ids, offs):
        calls.append((dev, len(offs) - 1))
        return model.encode(ids, offs)

    b = Batcher(encode_fn=enc, hidden=cfg["hidden"], devices=2, workers=1, max_rows=200, max_wait_us=5000)
    reqs = _requests(60, cfg["vocab"], seed=1)
    res, errs = _run_clients(b, reqs, 12)
    st = b.stats()
    b.close()
    assert all(e is None for e in errs)
    for r, got in zip(reqs, res):
        ids = np.concatenate([np.asarray(s, np.int32) for s in r])
        offs = np.concatenate([[0], np.cumsum([len(s) for s in r])]).astype(np.int64)
        assert np.array_equal(got.view(np.uint32), model.encode(ids, offs).view(np.uint32))
    assert st["requests"] == 60
    assert st["batches"] < 60  # requests were coalesced
    assert {d for d, _ in calls} == {0, 1}  # both devices took work


def test_failing_request_is_answered_alone(om):
    cfg, model = om

    def enc(dev, ids, offs):
        if (ids >= cfg["vocab"]).any():
            raise ValueError("out of vocabulary")
        return model.encode(ids, offs)

    b = Batcher(encode_fn=enc, hidden=cfg["hidden"], devices=1, workers=1, max_rows=10000, max_wait_us=20000)
    reqs = _requests(24, cfg["vocab"], seed=2)
    reqs[5] = [[1, 2, cfg["vocab"] + 7]]
    res, errs = _run_clients(b, reqs, 8)
    b.close()
    assert errs[5] is not None and res[5] is None
    assert all(e is None for i, e in enumerate(errs) if i != 5)


def test_no_wait_takes_only_queued_requests(om):
    """max_wait_us = 0 (the reference): a lone request leaves at once, alone."""
    cfg, model = om
    sizes = []

    def enc(dev, ids, offs):
        sizes.append(len(offs) - 1)
        return model.encode(ids, offs)

    b = Batcher(encode_fn=enc, hidden=cfg["hidden"], devices=1, workers=1, max_rows=512, max_wait_us=0)
    for r in _requests(5, cfg["vocab"], seed=3):
        b.encode(r)
    st = b.stats()
    b.close()
    assert st["batches"] == 5 and st["requests"] == 5
