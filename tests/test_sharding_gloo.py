"""Example sharding and the score all-gather across 2 CPU ranks (gloo), plus
a rank that fails before the collective: the survivor's collective ends with
an error inside the process-group timeout instead of hanging."""

import os
import socket
import traceback

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, n_total, fail_rank, results):
    import datetime
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=10))
    try:
        from cherimoya_b200.ism import gather_shards, shard_range
        lo, hi = shard_range(n_total, rank, world)
        if rank == fail_rank:
            raise RuntimeError("injected failure before the gather")
        # each rank's "scores": a deterministic function of the global index
        local = torch.arange(lo, hi, dtype=torch.float32).unsqueeze(1).repeat(1, 3) * 2.0
        full = gather_shards(local, n_total)
        expect = torch.arange(n_total, dtype=torch.float32).unsqueeze(1).repeat(1, 3) * 2.0
        results[rank] = bool(torch.equal(full, expect))
    except Exception:
        results[rank] = "error: " + traceback.format_exc().splitlines()[-1]
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(world, n_total, fail_rank=-1):
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    results = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, n_total, fail_rank, results))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert not p.is_alive()
        if p.is_alive():
            p.kill()
    return dict(results)


def test_gather_shards_two_ranks_uneven():
    res = _run(2, 7)
    assert res == {0: True, 1: True}


def test_gather_shards_two_ranks_even():
    res = _run(2, 256)
    assert res == {0: True, 1: True}


def test_failed_rank_surfaces_as_error_not_hang():
    res = _run(2, 10, fail_rank=1)
    assert isinstance(res[1], str) and "injected failure" in res[1]
    assert isinstance(res[0], str) and res[0].startswith("error")
