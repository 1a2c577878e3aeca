"""Batch sharding across ranks (one process per GPU, no collective on the hot
path), checked on CPU with world_size-2 gloo process groups: each rank runs
the decode step of its own rows, and the union over ranks equals the
single-process result, because nothing on the path mixes batch rows
(model/forecast.py, model/attention/sparse.py)."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from local_research_small_language_model_b200.sharding import batch_shard, max_over_ranks, sum_over_ranks
from oracle import sparda_oracle as O


def test_batch_shard_partitions_rows():
    for n in (0, 1, 5, 64, 513):
        for world in (1, 2, 3, 4, 8):
            parts = [batch_shard(n, r, world) for r in range(world)]
            assert parts[0][0] == 0 and parts[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(parts, parts[1:]))
            sizes = [b - a for a, b in parts]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        batch_shard(4, 2, 2)


def _decode_rows(rows, seed=3, L=700, hq=12, hkv=4):
    """One oracle decode step (selection + attention) for the given batch rows
    of a seeded global batch; every row draws its own inputs."""
    outs, sels = [], []
    for r in rows:
        g = np.random.default_rng(seed * 1000 + r)
        kd = g.standard_normal((1, hkv, L, 64))
        vd = g.standard_normal((1, hkv, L, 64))
        q = g.standard_normal((1, hq, 64))
        f = g.standard_normal((1, 1, hkv, 64))
        reps = O.compress_blocks(kd.transpose(0, 2, 1, 3), 64)
        sel, cnt = O.decode_select(f, reps, L, 64, 8, 1, hkv, "forecast", "absolute")
        outs.append(O.decode_attention(q, kd, vd, sel, cnt, L, 64))
        sels.append(sel)
    return np.concatenate(outs), np.concatenate(sels)


def _worker(rank, world, port, global_batch, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        a, b = batch_shard(global_batch, rank, world)
        out, sel = _decode_rows(range(a, b))
        slowest = max_over_ranks(float(rank + 1))
        rows = sum_over_ranks(float(b - a))
        q.put((rank, a, b, out, sel, slowest, rows))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("global_batch", [3, 4])
def test_two_rank_shards_reassemble_single_process_result(global_batch):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, global_batch, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    got.sort(key=lambda t: t[0])
    full_out, full_sel = _decode_rows(range(global_batch))
    out = np.concatenate([g[3] for g in got])
    sel = np.concatenate([g[4] for g in got])
    assert np.array_equal(sel, full_sel)
    np.testing.assert_array_equal(out, full_out)
    assert all(g[5] == float(world) for g in got)          # max over ranks
    assert all(g[6] == float(global_batch) for g in got)   # rows processed by the whole job
