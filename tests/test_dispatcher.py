"""Request-parallel dispatcher logic with fake engines (CPU), including host
fault injection and a 2-rank gloo check of the rank sharding."""
import os
import threading
import time

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from laya_b200.dispatcher import (B200Dispatcher, lpt_partition, group_by_bucket, shard_for_rank, shard_groups,
                                  group_cost, c4_step, bucket_of)


class FakeEngine:
    """Returns logits that encode (device, first token) so results can be traced."""

    def __init__(self, device, fail=False, delay=0.0):
        self.device, self.fail, self.delay = device, fail, delay
        self.calls = []
        self.closed = False

    def run_prepared(self, prepared):
        if self.fail:
            raise RuntimeError(f"injected failure on gpu {self.device}")
        time.sleep(self.delay)
        self.calls.append(len(prepared.items))
        k = max(2, max(len(it["markers"]) for it in prepared.items))
        logits = np.array([[float(it["ids"][0])] * k for it in prepared.items], np.float32)
        act = np.full((len(prepared.items), 2), float(self.device), np.float32)
        return logits, act, {}

    def close(self):
        self.closed = True


def items_of(lengths):
    return [{"ids": [i] * n, "markers": [1, 2], "qtype": 0} for i, n in enumerate(lengths)]


def test_lpt_partition_is_complete_disjoint_and_balanced():
    costs = [512, 480, 64, 64, 32, 256, 256, 128, 96, 512]
    bins = lpt_partition(costs, 3)
    flat = sorted(i for b in bins for i in b)
    assert flat == list(range(len(costs)))
    loads = [sum(costs[i] for i in b) for b in bins]
    assert max(loads) - min(loads) <= max(costs)
    assert lpt_partition(costs, 3) == bins          # deterministic


def test_group_by_bucket_respects_max_batch():
    items = items_of([30, 31, 33, 64, 65, 70, 500])
    groups = group_by_bucket(items, list(range(7)), tuple(range(32, 513, 32)), max_batch=2)
    assert groups == [(32, [0, 1]), (64, [2, 3]), (96, [4, 5]), (512, [6])]
    with pytest.raises(ValueError):
        bucket_of(513, (32, 512))


def test_results_come_back_in_input_order_from_every_gpu():
    engines = {}

    def factory(device, **_):
        engines[device] = FakeEngine(device)
        return engines[device]

    items = items_of([40, 300, 100, 500, 64, 200, 33, 480])
    with B200Dispatcher(devices=[0, 1, 2, 3], engine_factory=factory) as d:
        out = d.run_items(items)
    assert [float(lg[0]) for lg, _ in out] == [float(i) for i in range(len(items))]
    assert {int(a[0]) for _, a in out} == {0, 1, 2, 3}
    assert all(e.closed for e in engines.values())


def test_failed_gpu_is_marked_and_its_questions_rerun_elsewhere():
    def factory(device, **_):
        return FakeEngine(device, fail=(device == 1))

    items = items_of([100, 200, 300, 400])
    with B200Dispatcher(devices=[0, 1], engine_factory=factory) as d:
        out = d.run_items(items)
        assert d.healthy == {0: True, 1: False}
        assert all(int(a[0]) == 0 for _, a in out)
        assert [float(lg[0]) for lg, _ in out] == [0.0, 1.0, 2.0, 3.0]


def test_timeout_marks_gpu_unhealthy_and_errors_without_retry():
    def factory(device, **_):
        return FakeEngine(device, delay=(0.5 if device == 1 else 0.0))

    with B200Dispatcher(devices=[0, 1], engine_factory=factory, timeout=0.1, retry=False) as d:
        with pytest.raises(RuntimeError, match="worker failures"):
            d.run_items(items_of([100, 200, 300, 400]))
        assert d.healthy[1] is False


def test_one_deadline_for_the_whole_round():
    """Four slow GPUs each overrun the limit: the round still fails after about
    one timeout, not one timeout per GPU."""
    def factory(device, **_):
        return FakeEngine(device, delay=0.6)

    with B200Dispatcher(devices=[0, 1, 2, 3], engine_factory=factory, timeout=0.15, retry=False) as d:
        t0 = time.perf_counter()
        with pytest.raises(RuntimeError, match="worker failures"):
            d.run_items(items_of([100, 200, 300, 400]))
        assert time.perf_counter() - t0 < 0.45
        assert not any(d.healthy.values())


def test_close_does_not_wait_for_a_stuck_worker_and_keeps_its_engine():
    engines = {}
    release = threading.Event()

    class Stuck(FakeEngine):
        def run_prepared(self, prepared):
            release.wait(5)
            return super().run_prepared(prepared)

    def factory(device, **_):
        engines[device] = Stuck(device) if device == 1 else FakeEngine(device)
        return engines[device]

    d = B200Dispatcher(devices=[0, 1], engine_factory=factory, timeout=0.1)
    out = d.run_items(items_of([100, 200, 300, 400]))
    assert d.healthy == {0: True, 1: False} and all(int(a[0]) == 0 for _, a in out)
    t0 = time.perf_counter()
    d.close()
    assert time.perf_counter() - t0 < 1.0
    assert engines[0].closed and not engines[1].closed     # never freed under a running call
    release.set()


def test_readmit_puts_a_recovered_gpu_back_in_service():
    engines = {}

    def factory(device, **_):
        engines[device] = FakeEngine(device, fail=(device == 1))
        return engines[device]

    with B200Dispatcher(devices=[0, 1], engine_factory=factory) as d:
        d.run_items(items_of([100, 200]))
        assert d.healthy[1] is False
        assert d.readmit(items_of([40])) == []          # still failing: stays out
        engines[1].fail = False
        assert d.readmit(items_of([40])) == [1]
        out = d.run_items(items_of([100, 200, 300, 400]))
        assert {int(a[0]) for _, a in out} == {0, 1}


def test_all_gpus_failing_raises():
    with B200Dispatcher(devices=[0, 1], engine_factory=lambda dev, **_: FakeEngine(dev, fail=True)) as d:
        with pytest.raises(RuntimeError, match="no healthy GPU"):
            d.run_items(items_of([100, 200]))


def test_c4_step_is_seeded():
    a, b = c4_step(3, 1000), c4_step(3, 1000)
    assert [len(x["ids"]) for x in a] == [len(x["ids"]) for x in b] and len(a) == 64
    assert all(32 <= len(x["ids"]) <= 512 for x in a)


def test_group_sharding_is_complete_and_balanced():
    """Whole bucket groups per rank (what bench.py's C4 leg and the dispatcher
    use): every question exactly once, groups never split, loads within one
    group's cost of each other, the same answer on every call."""
    items = c4_step(7, 1000)
    for world in (1, 2, 4, 8):
        shards = shard_groups(items, world)
        assert len(shards) == world
        flat = sorted(i for shard in shards for _, idx in shard for i in idx)
        assert flat == list(range(len(items)))
        loads = [sum(group_cost(b, len(idx)) for b, idx in shard) for shard in shards]
        biggest = max(group_cost(b, len(idx)) for b, idx in group_by_bucket(items, list(range(64)),
                                                                          tuple(range(32, 513, 32)), 64))
        assert max(loads) - min(loads) <= biggest
        assert shard_groups(items, world) == shards
    assert group_cost(64, 1) == 64 + 2048 and group_cost(96, 5) == 96 * 8 + 2048


def _rank_main(rank, world, port, items, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import torch
    mine = sorted(i for _, idx in shard_groups(items, world)[rank] for i in idx)
    gathered = [None] * world
    dist.all_gather_object(gathered, mine)
    t = torch.tensor([float(rank + 1)])
    dist.all_reduce(t, op=dist.ReduceOp.MAX)     # max-over-ranks timing, as bench.py does
    if rank == 0:
        q.put((gathered, float(t.item())))
    dist.destroy_process_group()


def test_two_rank_sharding_over_gloo():
    items = c4_step(1, 1000)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + os.getpid() % 1000
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, items, q)) for r in range(2)]
    for p in procs:
        p.start()
    gathered, tmax = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    flat = sorted(i for shard in gathered for i in shard)
    assert flat == list(range(len(items))) and tmax == 2.0
    # the two ranks computed their shares independently and agree on the split
    want = [sorted(i for _, idx in shard for i in idx) for shard in shard_groups(items, 2)]
    assert gathered == want
