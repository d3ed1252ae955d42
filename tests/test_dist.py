"""CPU tests of the data-parallel host logic with gloo ranks (world size 2-3):
sharding, the logits all-gather, the max-over-ranks timing reduction, and a
failing rank that the others detect through the process-group timeout
instead of hanging. No GPU is touched."""

import os
import socket
import traceback

import pytest
import torch
import torch.multiprocessing as mp

from rpfq_review_b200 import dist as rdist


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _toy_logits(images: torch.Tensor) -> torch.Tensor:
    """Stand-in for the model: a deterministic per-image function."""
    g = torch.Generator().manual_seed(0)
    w = torch.randn(images[0].numel(), 10, generator=g)
    return images.reshape(images.shape[0], -1) @ w


def _worker(rank, world, port, mode, results, batch=12):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    try:
        rdist.init("gloo", timeout_s=10 if mode == "fail" else 60)
        g = torch.Generator().manual_seed(1)
        images = torch.randn(batch, 3, 4, 4, generator=g)
        s, e = rdist.shard_range(images.shape[0], world, rank)
        if mode == "fail" and rank == 1:
            raise RuntimeError("injected failure on rank 1 before the collective")
        local = _toy_logits(images[s:e])
        if mode == "reuse":
            # the gather object of a step loop: buffers allocated once, two calls
            gather = rdist.LogitsGather(batch, local.shape[1], world, rank)
            gather(local * 0)
            gathered = gather(local)
        else:
            gathered = rdist.gather_logits(local, batch)
        tmax = rdist.max_over_ranks(float(rank + 1), torch.device("cpu"))
        results[rank] = ("ok", torch.equal(gathered, _toy_logits(images)), tmax)
    except Exception as exc:  # reported to the parent
        results[rank] = ("error", type(exc).__name__, "".join(traceback.format_exception_only(exc)))
    finally:
        try:
            torch.distributed.destroy_process_group()
        except Exception:
            pass


def _run(world, mode, batch=12):
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    results = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, results, batch)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
            pytest.fail("a rank did not exit")
    return dict(results)


def test_shard_range_covers_batch():
    for n in (1, 7, 256, 2048):
        for world in (1, 2, 3, 8):
            spans = [rdist.shard_range(n, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [e - s for s, e in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        rdist.shard_range(8, 2, 2)


@pytest.mark.parametrize("world", [2, 3])
def test_gather_equals_single_process(world):
    res = _run(world, "ok")
    assert len(res) == world
    for r in range(world):
        status, equal, tmax = res[r]
        assert status == "ok" and equal
        assert tmax == float(world)  # max over ranks of (rank + 1)


@pytest.mark.parametrize("world,batch,mode", [(4, 10, "ok"), (3, 7, "reuse"), (2, 12, "reuse")])
def test_gather_uneven_shards(world, batch, mode):
    """A global batch that the world size does not divide (10 images over 4
    ranks: 3, 3, 2, 2) gathers into image order like the equal case."""
    res = _run(world, mode, batch)
    assert len(res) == world
    for r in range(world):
        status, equal, _ = res[r]
        assert status == "ok" and equal


def test_shard_sizes():
    assert rdist.shard_sizes(10, 4) == [3, 3, 2, 2]
    assert rdist.shard_sizes(256, 8) == [32] * 8
    assert rdist.shard_sizes(2048, 8) == [256] * 8


def test_failed_rank_is_detected_not_hung():
    res = _run(2, "fail")
    assert res[1][0] == "error" and "injected" in res[1][2]
    # the surviving rank's collective ends with an error (peer gone / timeout)
    assert res[0][0] == "error"
