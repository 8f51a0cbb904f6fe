"""Replica-per-GPU sharding exercised as 2 gloo ranks on CPU: every rank
embeds only its own batches (no data-path collective); a final all-gather
of the per-rank document counts (test bookkeeping only) shows that the
shards are disjoint and cover the corpus.  A rank that fails surfaces as an
error on the host without hanging the other rank."""
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from witchcraft_b200 import shard


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, fail_rank, q):
    import datetime
    import torch
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    try:
        lens = shard.config4_lengths(3000, seed=9)
        batches = shard.plan_batches(lens, 4096)
        mine = shard.assign_batches(batches, world)[rank]
        if rank == fail_rank:
            raise RuntimeError("injected worker failure")
        docs = np.concatenate([batches[i].docs for i in mine]) if mine else np.zeros(0, np.int64)
        counts = torch.zeros(3000, dtype=torch.int32)
        counts[torch.from_numpy(docs.astype(np.int64))] += 1
        dist.all_reduce(counts)
        q.put((rank, "ok", int(counts.min()), int(counts.max())))
    except Exception as e:  # noqa: BLE001
        q.put((rank, "err", str(e), 0))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(fail_rank):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, fail_rank, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return sorted(res)


def test_two_rank_shards_are_disjoint_and_complete():
    res = _run(fail_rank=-1)
    assert [r[1] for r in res] == ["ok", "ok"]
    assert all(r[2] == 1 and r[3] == 1 for r in res)


def test_failed_rank_surfaces_without_hanging():
    res = _run(fail_rank=1)
    assert res[1][1] == "err" and "injected" in res[1][2]
    assert res[0][1] == "err"  # the healthy rank's collective errors out instead of hanging
