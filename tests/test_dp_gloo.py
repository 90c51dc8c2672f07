"""Data-parallel host logic on CPU with world_size-2 gloo process groups (no GPU)."""
import datetime
import os
import socket

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

import dp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, global_batch, results, fail_rank):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    try:
        mine = dp.shard_requests(global_batch, rank, world)
        seeds = [dp.request_seed(1000, i) for i in mine]
        dp.barrier(dist)
        slowest = dp.max_over_ranks(dist, 10.0 * (rank + 1))
        total = dp.sum_over_ranks(dist, len(mine))
        if rank == fail_rank:
            raise RuntimeError("injected rank failure before the second barrier")
        try:
            dp.barrier(dist)
            results[rank] = ("ok", mine, seeds, slowest, total)
        except Exception as error:  # the peer never arrives: the short timeout ends the wait
            results[rank] = ("peer-failure-detected", type(error).__name__)
    except RuntimeError as error:
        results[rank] = ("raised", str(error))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(world, global_batch, fail_rank=-1):
    port = _free_port()
    manager = mp.get_context("spawn").Manager()
    results = manager.dict()
    mp.start_processes(_worker, args=(world, port, global_batch, results, fail_rank), nprocs=world,
                       join=True, start_method="spawn")
    return dict(results)


def test_shards_cover_requests_once():
    for world in (1, 2, 3, 8):
        for batch in (0, 1, 7, 8, 13):
            shards = [dp.shard_requests(batch, r, world) for r in range(world)]
            flat = [i for s in shards for i in s]
            assert flat == list(range(batch))
            assert max(map(len, shards)) - min(map(len, shards)) <= 1
    with pytest.raises(ValueError):
        dp.shard_requests(4, 2, 2)


def test_two_rank_gloo_group():
    out = _run(2, 8)
    assert out[0][0] == "ok" and out[1][0] == "ok"
    assert out[0][1] == [0, 1, 2, 3] and out[1][1] == [4, 5, 6, 7]
    assert set(out[0][2]).isdisjoint(out[1][2])
    assert out[0][3] == out[1][3] == 20.0  # max over ranks
    assert out[0][4] == out[1][4] == 8.0


def test_rank_failure_is_detected_not_hung():
    out = _run(2, 2, fail_rank=1)
    assert out[1][0] == "raised"
    assert out[0][0] == "peer-failure-detected"
