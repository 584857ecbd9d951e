"""Multi-GPU host logic on the CPU: two ranks (gloo) split a ragged batch
into cost-balanced contiguous ranges, each encodes its range and writes its
rows into a shared host output; the result equals the unsharded encode bit
for bit (sequences are independent: linalg/int8_test.go:149,
concurrency_test.go:12). The oracle stands in for each rank's GPU here; the
GPU path itself is covered by the gpu-marked encoder tests."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from indecis_b200 import shard
from indecis_b200 import synthetic as S


def test_shard_ranges_cover_and_balance():
    ids, offs = S.ids_varlen(101, 1, 512, 1000, seed=5)
    costs = shard.seq_costs(offs, 6, 3, 128, 256)
    for world in (1, 2, 3, 8):
        rs = shard.shard_ranges(offs, world, costs)
        assert rs[0][0] == 0 and rs[-1][1] == 101
        assert all(a[1] == b[0] for a, b in zip(rs, rs[1:]))
        loads = [costs[s0:s1].sum() for s0, s1 in rs]
        # contiguous split: no rank above its share plus the largest sequence
        assert max(loads) <= costs.sum() / world + costs.max() + 1e-6
    assert shard.shard_ranges(offs[:3], 8)[-1] == (2, 2)  # more ranks than sequences
    with pytest.raises(ValueError):
        shard.shard_ranges(offs, 0)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _cfg():
    return S.tiny(layers=2, hidden=64, heads=2, intermediate=96, vocab=200)


def _rank(rank, world, port, shm_name, rows, mode):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=60))
    import oracle
    cfg = _cfg()
    om = oracle.Model(cfg, S.weights(cfg, seed=3))
    ids, offs = S.ids_varlen(13, 1, 40, cfg["vocab"], seed=9)
    costs = shard.seq_costs(offs, cfg["layers"], cfg["global_every"], cfg["local_attention"], cfg["hidden"])
    # every rank derives the same split from the same offsets
    mine = torch.tensor(shard.shard_ranges(offs, world, costs), dtype=torch.int64)
    got = [torch.zeros_like(mine) for _ in range(world)]
    dist.all_gather(got, mine)
    assert all(torch.equal(g, mine) for g in got)
    out = shard.HostOutput(shm_name, rows, cfg["hidden"], create=False)
    m = 0 if mode == "pooled" else 1
    shard.encode_shard(lambda i, o: om.encode(i, o, mode=m), ids, offs, rank, world, out, costs, mode)
    dist.barrier()
    out.close()
    dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["pooled", "tokens"])
def test_two_ranks_gloo(mode):
    import oracle
    cfg = _cfg()
    ids, offs = S.ids_varlen(13, 1, 40, cfg["vocab"], seed=9)
    om = oracle.Model(cfg, S.weights(cfg, seed=3))
    ref = om.encode(ids, offs, mode=0 if mode == "pooled" else 1)
    name = f"ig_shard_test_{os.getpid()}_{mode}"
    out = shard.HostOutput(name, ref.shape[0], cfg["hidden"], create=True)
    try:
        out.array[:] = np.nan
        ctx = mp.get_context("spawn")
        port = _free_port()
        procs = [ctx.Process(target=_rank, args=(r, 2, port, name, ref.shape[0], mode)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
        assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
        assert np.array_equal(out.array.view(np.uint32), ref.view(np.uint32))
    finally:
        out.close()
