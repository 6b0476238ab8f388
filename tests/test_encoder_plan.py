"""Host logic of the data-parallel encoder step, on the CPU.

The allreduce plan must partition the gradient buffer (plus the loss/count
tail) exactly once, and the bucket-wise SUM allreduce must equal a plain
full allreduce -- checked with two gloo ranks (engine/step.py:62 psums the
loss, count and gradient tree together).
"""

import dataclasses
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from minifield_training_b200 import workloads
from minifield_training_b200.models import encoder as me
from minifield_training_b200.optimizers import adamw
from tests._util import run_ranks

TINY = dataclasses.replace(workloads.CONFIG5, global_batch=2, length=128, ffn=256,
                           layer_types=("conv", "full_attention", "conv"), vocab=1000)


@pytest.mark.parametrize("cfg", [workloads.CONFIG5, TINY], ids=["config5", "tiny"])
def test_plan_partitions_the_gradient_buffer(cfg):
    layout = adamw.Layout(me.inventory(cfg), me.arena_order(cfg))
    total = layout.n_train + 4
    plan = me.reduction_plan(layout, len(cfg.layer_types), total)
    cover = np.zeros(total, np.int32)
    for _, _, lo, hi in plan:
        cover[lo:hi] += 1
    assert (cover == 1).all()
    layers = [p for p in plan if p[0] == "layer"]
    assert [p[1] for p in layers] == list(reversed(range(len(cfg.layer_types))))
    # Fused groups are adjacent in the arena: gate|up and q|k|v.
    for i, kind in enumerate(cfg.layer_types):
        p = f"lfm2.layers.{i}."
        assert layout.offsets[p + "feed_forward.w3.weight"] == layout.offsets[p + "feed_forward.w1.weight"] + \
            layout.size(p + "feed_forward.w1.weight")
        if kind != "conv":
            q, k, v = (p + f"self_attn.{n}_proj.weight" for n in "qkv")
            assert layout.offsets[k] == layout.offsets[q] + layout.size(q)
            assert layout.offsets[v] == layout.offsets[k] + layout.size(k)


def test_matmul_parameter_count_matches_the_published_figure():
    assert workloads.encoder_matmul_params(workloads.CONFIG5) == 387_973_120


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    layout = adamw.Layout(me.inventory(TINY), me.arena_order(TINY))
    total = layout.n_train + 4
    plan = me.reduction_plan(layout, len(TINY.layer_types), total)
    g = torch.Generator().manual_seed(rank)
    flat = torch.randn(total, generator=g)
    expected = flat.clone()
    dist.all_reduce(expected)
    events = []

    def reduce_range(lo, hi):
        events.append(("reduce", lo, hi))
        dist.all_reduce(flat[lo:hi])  # the bucket, in place (a view of the flat buffer)

    red = me.BucketReducer(plan, reduce_range, before=lambda: events.append(("before",)),
                           after=lambda: events.append(("after",)))
    for i in reversed(range(len(TINY.layer_types))):
        red.layer_done(i)
    red.finish()
    # Every reduction follows its ordering hook; the closing hook comes last, once.
    assert events[-1] == ("after",) and events.count(("after",)) == 1
    assert all(events[k] == ("before",) for k in range(0, len(events) - 1, 2))
    reduced = sorted((e[1], e[2]) for e in events if e[0] == "reduce")
    assert reduced[0][0] == 0 and reduced[-1][1] == total
    assert all(a[1] == b[0] for a, b in zip(reduced, reduced[1:]))  # the ranges tile [0, total)
    out[rank] = float((flat - expected).abs().max())
    dist.destroy_process_group()


def test_bucketed_allreduce_equals_full_allreduce_on_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    port = 29400 + os.getpid() % 500
    run_ranks(ctx, _worker, [(r, 2, port, out) for r in range(2)], 120)
    assert out[0] == 0.0 and out[1] == 0.0


@pytest.mark.parametrize("n", [1, 3, 4, 17, 1000, 388_000_001])
@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_optimizer_slices_partition_the_range(n, world):
    """The sharded AdamW slices: equal 4-aligned slices covering [0, n) once (empty ones past n)."""
    slices = [adamw.shard_slices(n, world, r) for r in range(world)]
    per = slices[0][2]
    assert per % 4 == 0 and per * world >= n and all(s[2] == per for s in slices)
    covered = 0
    for r, (lo, hi, _) in enumerate(slices):
        assert (lo % 4 == 0 or lo == hi) and lo <= hi and lo == min(r * per, n)
        assert hi == min(lo + per, n)
        covered += hi - lo
    assert covered == n


def test_sharded_master_arena_holds_the_all_gather():
    layout = adamw.Layout(me.inventory(TINY), me.arena_order(TINY))
    for world in (1, 2, 8):
        per = adamw.shard_slices(layout.n_train, world, 0)[2]
        assert adamw.sharded_master_elements(layout, world) >= max(layout.n_total, per * world)


def _leaf_ranges(layout):
    return [(layout.offsets[n], layout.offsets[n] + layout.size(n)) for n in layout.trainable]


@pytest.mark.parametrize("cfg", [workloads.CONFIG5, TINY], ids=["config5", "tiny"])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_owner_ranges_tile_the_trainable_arena_at_bucket_starts(cfg, world):
    """Sharded optimizer: contiguous owned ranges tiling [0, n_train), cut only at bucket starts
    (so no leaf is split between owners), and within one bucket of an equal share."""
    layout = adamw.Layout(me.inventory(cfg), me.arena_order(cfg))
    plan = me.reduction_plan(layout, len(cfg.layer_types), layout.n_train + 4)
    owners = me.owner_ranges(plan, layout.n_train, world)
    assert len(owners) == world and owners[0][0] == 0 and owners[-1][1] == layout.n_train
    assert all(a[1] == b[0] for a, b in zip(owners, owners[1:]))
    assert all(lo <= hi and lo % 4 == 0 for lo, hi in owners)
    for lo, hi in _leaf_ranges(layout):
        assert sum(1 for a, b in owners if a <= lo and hi <= b) == 1, (lo, hi)
    if cfg is workloads.CONFIG5 and world in (2, 4, 8):
        biggest = max(hi - lo for kind, _, lo, hi in plan if kind == "layer")
        assert max(hi - lo for lo, hi in owners) <= layout.n_train / world + biggest


@pytest.mark.parametrize("world", [1, 2, 8])
def test_broadcast_plan_sends_every_master_once_from_its_owner(world):
    layout = adamw.Layout(me.inventory(workloads.CONFIG5), me.arena_order(workloads.CONFIG5))
    n_layers = len(workloads.CONFIG5.layer_types)
    plan = me.reduction_plan(layout, n_layers, layout.n_train + 4)
    owners = me.owner_ranges(plan, layout.n_train, world)
    bplan = me.broadcast_plan(plan, layout.n_train, owners)
    assert [k for k, _ in bplan] == ["vectors"] + [("layer", i) for i in range(n_layers)] + ["head"]
    cover = np.zeros(layout.n_train, np.int8)
    for _, pieces in bplan:
        for lo, hi, r in pieces:
            assert owners[r][0] <= lo < hi <= owners[r][1]
            cover[lo:hi] += 1
    assert cover.max() == 1
    for lo, hi in _leaf_ranges(layout):
        assert (cover[lo:hi] == 1).all(), (lo, hi)


def _owner_worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    layout = adamw.Layout(me.inventory(TINY), me.arena_order(TINY))
    total = layout.n_train + 4
    plan = me.reduction_plan(layout, len(TINY.layer_types), total)
    owners = me.owner_ranges(plan, layout.n_train, world)
    g = torch.Generator().manual_seed(rank)
    flat = torch.randn(total, generator=g)
    expected = flat.clone()
    dist.all_reduce(expected)

    def reduce_range(lo, hi):
        for x, y, root in me.owner_reductions(lo, hi, owners, layout.n_train):
            if root is None:
                dist.all_reduce(flat[x:y])
            else:
                buf = flat[x:y].clone()
                dist.reduce(buf, dst=root)
                if rank == root:
                    flat[x:y] = buf

    red = me.BucketReducer(plan, reduce_range)
    for i in reversed(range(len(TINY.layer_types))):
        red.layer_done(i)
    red.finish()
    lo, hi = owners[rank]
    out[rank] = (float((flat[lo:hi] - expected[lo:hi]).abs().max()) if hi > lo else 0.0,
                 float((flat[layout.n_train:] - expected[layout.n_train:]).abs().max()))
    dist.destroy_process_group()


def test_owner_reductions_give_each_owner_the_full_sum_on_three_gloo_ranks():
    """Sharded optimizer: reducing every bucket to its owners (and allreducing the loss/count tail)
    leaves each rank's owned range, and the tail, equal to a full allreduce."""
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    port = 29900 + os.getpid() % 90
    run_ranks(ctx, _owner_worker, [(r, 3, port, out) for r in range(3)], 120)
    for r in range(3):
        assert out[r][0] < 1e-5 and out[r][1] < 1e-5, out[r]
