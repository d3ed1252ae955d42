"""CPU tests of bench.py's strong-scaling plan: every rank draws the same
seeded global batch and keeps the slice dist.shard_range gives it, so the
shards put back together are the 1-GPU batch for any world size (uneven
splits included), and --batch switches to the weak mode."""

import argparse

import torch

import bench
from rpfq_review_b200.vit import VIT_B16, VIT_L16


def _args(**kw):
    a = argparse.Namespace(batch=None, global_batch=None)
    a.__dict__.update(kw)
    return a


def test_default_global_batches():
    assert bench.batch_plan(_args(), VIT_B16, 8, 0) == (256, (0, 32), "strong")
    assert bench.batch_plan(_args(), VIT_L16, 8, 7) == (2048, (1792, 2048), "strong")
    assert bench.batch_plan(_args(batch=32), VIT_B16, 4, 1) == (128, (32, 64), "weak")
    assert bench.batch_plan(_args(global_batch=10), VIT_B16, 4, 1) == (10, (3, 6), "strong")


def test_shards_reassemble_the_global_batch():
    cfg = VIT_B16
    gb = 12
    whole = bench.global_images(cfg, gb, 0, gb, "cpu")
    for world in (1, 2, 3, 5, 8):
        parts = []
        for rank in range(world):
            _, (s, e), _ = bench.batch_plan(_args(global_batch=gb), cfg, world, rank)
            parts.append(bench.global_images(cfg, gb, s, e, "cpu"))
        assert torch.equal(torch.cat(parts), whole)
