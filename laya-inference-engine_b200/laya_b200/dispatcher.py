"""Request-parallel dispatch of decision questions over 1-8 GPUs of one node.

The reference serves one GPU per engine behind a lock
(``src/laya_blackwell/engine.py:84,192``) and has no multi-GPU path; its
multi-stream ``StreamService`` prototype (``experiments/latency/serving``)
overlaps independent requests.  Here every GPU holds its own weight replica,
CUDA graphs and pinned buffers (one ``B200Engine`` per device, driven by its
own worker thread: ctypes releases the GIL inside the native forward), and
independent questions are partitioned across GPUs:

* questions that share a sequence bucket form one batched forward (at most
  ``max_batch``, batch padded to a power of two, as ``BlackwellEngine._shape``);
* each group is priced at its padded tokens plus a fixed per-forward cost
  (``group_cost``), and whole groups are assigned longest-first to the
  least-loaded GPU (LPT), so a GPU runs a few full batches rather than many
  one-question forwards.

There is no collective anywhere: results return to the caller's thread.
Failure handling is on the host: a worker that raises, or that has not
finished when the round's single deadline (``timeout`` seconds after the round
was dispatched) passes, marks its GPU unhealthy, and its questions are re-run
on the healthy GPUs (``retry=True``) or reported as errors.  ``readmit()``
probes unhealthy GPUs whose worker has returned and puts them back in service
when a probe request succeeds.  ``close()`` never waits on a worker that is
still stuck: its pool is shut down without waiting and its engine is left open
(closing it under a running native call would free memory the call uses).
"""
from concurrent.futures import ThreadPoolExecutor, wait as futures_wait
import threading

import numpy as np

from .engine import request_from_items


def bucket_of(length, buckets):
    for b in buckets:
        if length <= b:
            return b
    raise ValueError(f"sequence of {length} tokens exceeds the largest bucket {buckets[-1]}")


def lpt_partition(costs, parts):
    """Longest-processing-time-first assignment of items to `parts` bins.

    Deterministic (ties broken by item index, then bin index), so every rank of
    a multi-process job computes the same partition without communicating.
    Returns a list of index lists, one per bin."""
    if parts < 1:
        raise ValueError("parts must be positive")
    order = sorted(range(len(costs)), key=lambda i: (-costs[i], i))
    load = [0] * parts
    bins = [[] for _ in range(parts)]
    for i in order:
        j = min(range(parts), key=lambda p: (load[p], p))
        bins[j].append(i)
        load[j] += costs[i]
    for b in bins:
        b.sort()
    return bins


def group_by_bucket(items, indices, buckets, max_batch):
    """Batches of item indices that share a sequence bucket (<= max_batch each)."""
    groups = {}
    for i in indices:
        groups.setdefault(bucket_of(len(items[i]["ids"]), buckets), []).append(i)
    out = []
    for bucket in sorted(groups):
        idx = groups[bucket]
        for s in range(0, len(idx), max_batch):
            out.append((bucket, idx[s:s + max_batch]))
    return out


class B200Dispatcher:
    """Serve independent questions on several GPUs, one engine replica each."""

    def __init__(self, devices=(0,), *, engine_factory=None, timeout=None, retry=True,
                 sequence_buckets=tuple(range(32, 513, 32)), max_batch=64, **engine_kwargs):
        if not devices:
            raise ValueError("at least one device is required")
        self.devices = list(devices)
        self.timeout, self.retry = timeout, retry
        self.buckets = tuple(sorted(sequence_buckets))
        self.max_batch = max_batch
        if engine_factory is None:
            from .engine import B200Engine

            def engine_factory(device, **kw):
                return B200Engine(device=device, sequence_buckets=self.buckets, max_questions=max_batch, **kw)
        self.engines = {}
        with ThreadPoolExecutor(max_workers=len(self.devices)) as ex:
            futs = {d: ex.submit(engine_factory, d, **engine_kwargs) for d in self.devices}
            for d, f in futs.items():
                self.engines[d] = f.result()
        self.pools = {d: ThreadPoolExecutor(max_workers=1, thread_name_prefix=f"laya-gpu{d}")
                      for d in self.devices}
        self.healthy = {d: True for d in self.devices}
        self.inflight = {d: None for d in self.devices}   # last future submitted to each worker
        self.lock = threading.Lock()
        self.closed = False

    def _run_batches(self, device, items, batches):
        eng = self.engines[device]
        out = {}
        for _, idx in batches:
            logits, act, _ = eng.run_prepared(request_from_items([items[i] for i in idx]))
            for row, i in enumerate(idx):
                k = len(items[i]["markers"])
                out[i] = (logits[row, :max(k, 1)].copy(), act[row].copy())
        return out

    def run_items(self, items):
        """Logits [k_i] and act [2] per item, in input order.

        Raises RuntimeError when an item could not be served on any GPU."""
        if self.closed:
            raise RuntimeError("Dispatcher is closed")
        if not items:
            return []
        results = {}
        pending = list(range(len(items)))
        errors = {}
        while pending:
            with self.lock:
                alive = [d for d in self.devices if self.healthy[d]]
            if not alive:
                raise RuntimeError(f"no healthy GPU left; {len(pending)} questions unserved: {errors}")
            # whole bucket groups per GPU (LPT by estimated forward cost)
            groups = split_for_balance(group_by_bucket(items, pending, self.buckets, self.max_batch), len(alive))
            shards = lpt_partition([group_cost(b, len(g)) for b, g in groups], len(alive))
            futs = {}
            for d, shard in zip(alive, shards):
                batches = [groups[j] for j in shard]
                idx = sorted(i for _, g in batches for i in g)
                if idx:
                    fut = self.pools[d].submit(self._run_batches, d, items, batches)
                    self.inflight[d] = fut
                    futs[d] = (idx, fut)
            # one deadline for the whole round, however many GPUs take part
            futures_wait([f for _, f in futs.values()], timeout=self.timeout)
            failed = []
            for d, (idx, fut) in futs.items():
                exc = None
                if not fut.done():
                    exc = TimeoutError(f"gpu {d} did not finish within {self.timeout} s")
                elif fut.exception() is not None:
                    exc = fut.exception()
                if exc is None:
                    results.update(fut.result())
                    continue
                with self.lock:
                    self.healthy[d] = False
                errors[d] = repr(exc)
                failed.extend(idx)
            if failed and not self.retry:
                raise RuntimeError(f"GPU worker failures: {errors}")
            pending = sorted(failed)
        return [results[i] for i in range(len(items))]

    def _idle(self, device):
        fut = self.inflight[device]
        return fut is None or fut.done()

    def readmit(self, probe_items, timeout=None):
        """Probe every unhealthy GPU whose worker has returned with
        `probe_items` (a small request) and mark it healthy again when the probe
        succeeds.  Returns the devices put back in service."""
        if self.closed:
            raise RuntimeError("Dispatcher is closed")
        back = []
        for d in self.devices:
            with self.lock:
                if self.healthy[d] or not self._idle(d):
                    continue
            batches = group_by_bucket(probe_items, list(range(len(probe_items))), self.buckets, self.max_batch)
            fut = self.pools[d].submit(self._run_batches, d, probe_items, batches)
            self.inflight[d] = fut
            futures_wait([fut], timeout=timeout if timeout is not None else self.timeout)
            if fut.done() and fut.exception() is None:
                with self.lock:
                    self.healthy[d] = True
                back.append(d)
        return back

    def close(self):
        if self.closed:
            return
        self.closed = True
        for d in self.devices:
            if self._idle(d):
                self.pools[d].shutdown(wait=True)
                self.engines[d].close()
            else:  # a worker still inside a call: do not wait for it, do not free its engine
                self.pools[d].shutdown(wait=False, cancel_futures=True)

    def __enter__(self):
        return self

    def __exit__(self, *_):
        self.close()


def shard_for_rank(items, world, rank, buckets=tuple(range(32, 513, 32))):
    """The items one rank of a multi-process job serves (same LPT on every rank)."""
    costs = [bucket_of(len(it["ids"]), buckets) for it in items]
    return lpt_partition(costs, world)[rank]


# Fixed cost of one batched forward in token-equivalents: a short forward is
# bound by its dependent launches, not by its tokens (a 1 x 64 bf16 forward
# takes as long as ~2k tokens of batched FP8 work on a B200).
FORWARD_OVERHEAD_TOKENS = 2048


def group_cost(bucket, batch):
    """Estimated cost of one bucket group: padded tokens plus the fixed
    per-forward overhead (the batch pads to a power of two, as
    BlackwellEngine._shape does)."""
    padded = 1 << (batch - 1).bit_length()
    return bucket * padded + FORWARD_OVERHEAD_TOKENS


def shard_groups(items, world, buckets=tuple(range(32, 513, 32)), max_batch=64):
    """Whole bucket groups per rank: every rank forms the same groups (by
    sequence bucket, at most max_batch each) and takes its LPT share of them
    by group_cost, so a rank runs a few full batches rather than many
    one-question forwards.  Returns, per rank, the list of (bucket, indices)."""
    groups = split_for_balance(group_by_bucket(items, list(range(len(items))), buckets, max_batch), world)
    costs = [group_cost(b, len(idx)) for b, idx in groups]
    return [[groups[g] for g in part] for part in lpt_partition(costs, world)]


def split_for_balance(groups, parts):
    """Split the most expensive group (at its largest power of two below its
    size, so neither half pads) while it costs more than an even share of the
    work over `parts` GPUs; deterministic.  One GPU keeps the groups whole."""
    groups = list(groups)
    if parts <= 1:
        return groups
    while True:
        costs = [group_cost(b, len(idx)) for b, idx in groups]
        worst = max(range(len(groups)), key=lambda g: (costs[g], -g))
        bucket, idx = groups[worst]
        if len(idx) == 1 or costs[worst] <= sum(costs) / parts:
            return groups
        half = 1 << ((len(idx) - 1).bit_length() - 1)
        groups[worst:worst + 1] = [(bucket, idx[:half]), (bucket, idx[half:])]


def c4_step(seed, vocab, questions=64, lo=32, hi=512):
    """`questions` questions, lengths uniform in [lo, hi],
    seeded mix of question types."""
    from .workload import synthetic_items, mixed_kinds
    rng = np.random.Generator(np.random.PCG64(seed))
    lengths = rng.integers(lo, hi + 1, size=questions).tolist()
    return synthetic_items(lengths, mixed_kinds(questions, seed), seed=seed, vocab=vocab)
