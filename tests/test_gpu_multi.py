"""Several GPUs in one process: the batch sharded across devices behind the C ABI.

ig_model_create_multi replicates the weights on every listed GPU; a host call
splits its sequences into contiguous cost-balanced ranges, one per GPU, and
each range writes its rows into its slice of the caller's output. Sequences
are independent (linalg/int8_test.go:149, concurrency_test.go:51-60), so the
result must equal one GPU's bit for bit. The batcher over one model per GPU
(WithBatching, batch.go:24-81) is checked the same way with its models on two
different devices. Each test also exercises every large-shared-memory kernel
on the second GPU, whose per-device launch attributes must be set there too.

These tests need two GPUs and skip otherwise; they use plain launches on each
device, no peer memory.
"""
import threading

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")


def _cfg():
    from indecis_b200 import synthetic as S
    return S.tiny(layers=3, hidden=256, heads=4, intermediate=384, vocab=2000)


def test_multi_device_model_matches_one_device(igdev):
    _two_gpus()
    from indecis_b200 import synthetic as S
    from indecis_b200.model import Config, Head, Model
    cfg = _cfg()
    W = S.weights(cfg, seed=42)
    one = Model.from_arrays(Config.from_dict(cfg), W, device=0)
    two = Model.from_arrays(Config.from_dict(cfg), W, device=[1, 0])
    assert two.device_count() == 2
    assert two.replica(0)[1] == 1 and two.replica(1)[1] == 0
    heads = [Head(h["name"], h["kind"], h["w"], h["b"]) for h in S.heads(cfg["hidden"])]
    one.SetHeads(heads)
    two.SetHeads(heads)
    # 200 sequences of 1..300 tokens: about 30k rows, enough for two shards
    # (ragged, so the cost split does not fall on equal counts), and a batch
    # of 128-token sequences.
    for ids, offs in (S.ids_varlen(200, 1, 300, cfg["vocab"], seed=9),
                      S.ids_varlen(160, 128, 128, cfg["vocab"], seed=10)):
        assert offs[-1] >= 2 * 8192
        for mode in ("pooled", "tokens"):
            f = (lambda m: m.EncodeSeqs((ids, offs))) if mode == "pooled" else (lambda m: m.EncodeTokens((ids, offs)))
            a, b = f(one), f(two)
            assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), mode
        za, _ = one.Logits((ids, offs))
        zb, _ = two.Logits((ids, offs))
        assert len(za) == len(heads)
        for x, y in zip(za, zb):
            assert np.array_equal(np.ascontiguousarray(x).view(np.uint64), np.ascontiguousarray(y).view(np.uint64))
    one.close()
    two.close()


def test_multi_device_concurrent_calls_and_errors(igdev):
    _two_gpus()
    from indecis_b200 import synthetic as S
    from indecis_b200.model import Config, ModernBertError, Model
    cfg = _cfg()
    W = S.weights(cfg, seed=7)
    one = Model.from_arrays(Config.from_dict(cfg), W, device=0)
    two = Model.from_arrays(Config.from_dict(cfg), W, device=[0, 1])
    batches = [S.ids_varlen(int(n), 1, 200, cfg["vocab"], seed=int(s)) for n, s in zip([3, 40, 150, 7, 90, 120], range(6))]
    want = [one.EncodeSeqs(b) for b in batches]
    got = [None] * len(batches)

    def run(i):
        got[i] = two.EncodeSeqs(batches[i])

    ts = [threading.Thread(target=run, args=(i,)) for i in range(len(batches))]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    for a, b in zip(want, got):
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    # An out-of-vocabulary id in the second shard fails the whole call with
    # the reference's message (infer.go:310-312), naming the first bad id.
    ids, offs = S.ids_varlen(160, 128, 128, cfg["vocab"], seed=11)
    ids = ids.copy()
    ids[int(offs[150]) + 3] = cfg["vocab"] + 5
    ids[int(offs[120])] = cfg["vocab"] + 1
    with pytest.raises(ModernBertError, match=f"id {cfg['vocab'] + 1} out of vocabulary"):
        two.EncodeSeqs((ids, offs))
    one.close()
    two.close()


def test_batcher_on_two_devices(igdev):
    _two_gpus()
    from indecis_b200 import synthetic as S
    from indecis_b200.batch import Batcher
    from indecis_b200.model import Config, Model
    cfg = S.tiny(layers=3, hidden=128, heads=2, intermediate=192, vocab=900)
    W = S.weights(cfg, seed=17)
    models = [Model.from_arrays(Config.from_dict(cfg), W, device=d) for d in (0, 1)]
    b = Batcher(models, workers=2, max_rows=2048, max_wait_us=2000)
    rng = np.random.default_rng(8)
    reqs = [[rng.integers(0, 900, int(rng.integers(1, 200))).tolist() for _ in range(int(rng.integers(1, 5)))]
            for _ in range(120)]
    res = [None] * len(reqs)

    def client(t):
        for i in range(t, len(reqs), 12):
            res[i] = b.encode(reqs[i])

    ts = [threading.Thread(target=client, args=(t,)) for t in range(12)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    b.close()
    for r, got in zip(reqs, res):
        assert np.array_equal(got.view(np.uint32), models[0].EncodeSeqs(r).view(np.uint32))
    for m in models:
        m.close()
