"""Batch-sharding bookkeeping on CPU ranks (gloo, world size 2): balanced
shards, rank-ordered logits gather, max-over-ranks timing, and a rank that
fails before the collective being reported (not hung) on the other rank."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from intp_preliminary_b200.sharding import (
    RankContext,
    gather_to_main,
    init_from_env,
    max_over_ranks,
    shard_bounds,
    shutdown,
)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_bounds_cover_the_batch_exactly():
    for batch in (0, 1, 7, 256, 1023):
        for world in (1, 2, 3, 8):
            spans = [shard_bounds(batch, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == batch
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [stop - start for start, stop in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_bounds(4, 2, 2)


def _worker(rank: int, world: int, port: int, batch: int, fail_rank: int, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    ctx = init_from_env("gloo", timeout_s=20.0)
    try:
        start, stop = shard_bounds(batch, world, rank)
        images = torch.arange(batch * 3, dtype=torch.float32).reshape(batch, 3)[start:stop]
        logits = images * 2.0 + 1.0  # stand-in for the model forward
        if rank == fail_rank:
            raise RuntimeError("injected failure before the logits gather")
        gathered = gather_to_main(logits, ctx, batch)
        slowest = max_over_ranks(float(rank + 1) * 1.5, ctx)
        results[rank] = ("ok", None if gathered is None else gathered.tolist(), slowest)
    except Exception as exc:  # reported back to the parent
        results[rank] = ("error", repr(exc), None)
    finally:
        try:
            shutdown(ctx)
        except Exception:
            pass


def _run(world: int, batch: int, fail_rank: int = -1):
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, batch, fail_rank, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
            pytest.fail("a rank did not finish within 120 s")
    return dict(results)


@pytest.mark.parametrize("batch", [8, 7])
def test_gather_and_max_over_two_gloo_ranks(batch):
    res = _run(2, batch)
    assert res[0][0] == "ok" and res[1][0] == "ok", res
    expected = (torch.arange(batch * 3, dtype=torch.float32).reshape(batch, 3) * 2.0 + 1.0).tolist()
    assert res[0][1] == expected
    assert res[1][1] is None
    assert res[0][2] == 3.0 and res[1][2] == 3.0


def test_failed_rank_is_reported_not_hung():
    res = _run(2, 8, fail_rank=1)
    assert res[1][0] == "error" and "injected failure" in res[1][1]
    assert res[0][0] == "error", res  # the surviving rank's gather errors out instead of waiting forever


def test_single_process_context_needs_no_group():
    ctx = RankContext(0, 1, 0, torch.device("cpu"))
    t = torch.ones(3, 2)
    assert gather_to_main(t, ctx, 3) is t
    assert max_over_ranks(2.5, ctx) == 2.5
