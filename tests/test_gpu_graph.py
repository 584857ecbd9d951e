"""Repeated host calls replayed from a recorded CUDA graph.

A host call of at most 16384 tokens whose offsets, mode and outputs repeat the
previous call's on the same workspace runs its kernels as one graph launch
(recorded on the second sight, replayed after that). The reference has no such
mechanism, so what is checked is that it changes nothing: every call bit for
bit against the oracle with new ids each time, before and after the graph is
recorded, through the pooled, per-token and head-logit entry points, after a
change of heads (the graph is recorded again) and with another batch shape in
between; and that the graphs were in fact recorded and replayed."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _bits(a):
    return np.ascontiguousarray(a).view(np.uint64 if a.dtype == np.float64 else np.uint32)


def _graph_counts():
    from indecis_b200 import _capi
    rep = _capi.profile_report()
    return rep["graphs_recorded"], rep["graph_runs"]


def test_repeated_shapes_replay_bitexact(igdev, oracle_lib):
    import oracle
    from indecis_b200 import synthetic as S
    from indecis_b200.model import Config, Head, Model
    cfg = S.tiny(layers=3, hidden=256, heads=4, intermediate=384, vocab=2000)
    W = S.weights(cfg, seed=11, gamma_noise=0.1)
    om, gm = oracle.Model(cfg, W), Model.from_arrays(Config.from_dict(cfg), W)
    rng = np.random.default_rng(5)
    lens = [128, 77, 1, 128, 0, 30, 64]
    offs = np.concatenate([[0], np.cumsum(lens)]).astype(np.int64)

    def ids():
        return rng.integers(4, cfg["vocab"], int(offs[-1])).astype(np.int32)

    rec0, run0 = _graph_counts()
    # Pooled: first sight, recording, two replays.
    for _ in range(4):
        x = ids()
        assert np.array_equal(_bits(gm.EncodeSeqs((x, offs))), _bits(om.encode(x, offs, threads=8)))
    rec1, run1 = _graph_counts()
    assert rec1 - rec0 == 1 and run1 - run0 == 3
    # Per-token states: another key.
    for _ in range(3):
        x = ids()
        assert np.array_equal(_bits(gm.EncodeTokens((x, offs))), _bits(om.encode(x, offs, mode=1, threads=8)))
    # A different shape in between, then the first shape again (recorded anew:
    # the workspace holds one graph).
    x2, offs2 = S.ids_varlen(5, 1, 120, cfg["vocab"], seed=3)
    assert np.array_equal(_bits(gm.EncodeSeqs((x2, offs2))), _bits(om.encode(x2, offs2, threads=8)))
    for _ in range(3):
        x = ids()
        assert np.array_equal(_bits(gm.EncodeSeqs((x, offs))), _bits(om.encode(x, offs, threads=8)))
    # Head logits, then new heads: the graph of the old heads is not replayed.
    for seed, shift in ((1, 0.01), (2, -0.03)):
        heads = [Head(h["name"], h["kind"], h["w"], h["b"] + np.float32(shift))
                 for h in S.heads(cfg["hidden"], seed=seed)]
        gm.SetHeads(heads)
        for _ in range(3):
            x = ids()
            logits, _ = gm.Logits((x, offs))
            pooled = om.encode(x, offs, threads=8)
            tokens = om.encode(x, offs, mode=1, threads=8)
            for h, z in zip(heads, logits):
                ref = oracle.head_logits(h.w, h.b, tokens if h.kind == "spans" else pooled)
                assert np.array_equal(_bits(z), _bits(ref)), (seed, h.name)
    # Recorded: tokens, pooled again, logits, logits after the heads changed
    # (the key was seen already, so at once); launched: each recording and
    # the replays after it.
    rec2, run2 = _graph_counts()
    assert rec2 - rec1 == 4 and run2 - run1 == 2 + 2 + 2 + 3
    gm.close()


def test_replay_reports_out_of_vocabulary(igdev, oracle_lib):
    """An id check failing on a call whose shape has a recorded graph is still
    an error before any work, and the next call replays correctly."""
    import oracle
    from indecis_b200 import synthetic as S
    from indecis_b200.model import Config, Model, ModernBertError
    cfg = S.tiny(layers=2, hidden=128, heads=2, intermediate=256, vocab=500)
    W = S.weights(cfg, seed=2)
    om, gm = oracle.Model(cfg, W), Model.from_arrays(Config.from_dict(cfg), W)
    x, offs = S.ids_fixed(4, 32, cfg["vocab"], seed=8)
    ref = om.encode(x, offs)
    for _ in range(3):
        assert np.array_equal(_bits(gm.EncodeSeqs((x, offs))), _bits(ref))
    bad = x.copy()
    bad[40] = 500
    with pytest.raises(ModernBertError, match="out of vocabulary"):
        gm.EncodeSeqs((bad, offs))
    assert np.array_equal(_bits(gm.EncodeSeqs((x, offs))), _bits(ref))
    gm.close()


def test_concurrent_callers_record_and_replay(igdev, oracle_lib):
    """Eight threads calling on one model with batches of one shape: each
    call takes its own workspace, so the graphs are recorded concurrently on
    several streams and replayed; every result bit for bit as the oracle's."""
    import threading

    import oracle
    from indecis_b200 import synthetic as S
    from indecis_b200.model import Config, Model
    cfg = S.tiny(layers=2, hidden=256, heads=4, intermediate=384, vocab=3000)
    W = S.weights(cfg, seed=19)
    om, gm = oracle.Model(cfg, W), Model.from_arrays(Config.from_dict(cfg), W)
    _, offs = S.ids_fixed(6, 96, cfg["vocab"], seed=1)
    rng = np.random.default_rng(9)
    batches = [rng.integers(4, cfg["vocab"], int(offs[-1])).astype(np.int32) for _ in range(12)]
    refs = [om.encode(x, offs, threads=4) for x in batches]
    rec0, run0 = _graph_counts()
    errors = []

    def work(t):
        try:
            for i in range(6):
                k = (t + i) % len(batches)
                got = gm.EncodeSeqs((batches[k], offs))
                if not np.array_equal(_bits(got), _bits(refs[k])):
                    errors.append((t, i))
        except Exception as e:  # reported below, in the main thread
            errors.append((t, repr(e)))

    ths = [threading.Thread(target=work, args=(t,)) for t in range(8)]
    [t.start() for t in ths]
    [t.join() for t in ths]
    assert not errors, errors[:5]
    rec1, run1 = _graph_counts()
    assert rec1 > rec0 and run1 - run0 >= rec1 - rec0
    gm.close()
