"""The ``b200`` engine mode: BlackwellEngine's contract over the native library.

Mirrors ``src/laya_blackwell/engine.py``:

* constructor kwargs and their validation (``engine.py:74-104``), plus
  ``precision`` in {bf16, fp8, nvfp4} and the seeded-weight options;
* ``_shape`` / ``_graph_key`` / ``_fill`` bucketing and padding semantics
  (``engine.py:112-153``);
* an LRU of captured CUDA-graph slots (``engine.py:161-187``);
* ``run_prepared`` returning owned numpy arrays under one lock
  (``engine.py:189-214``), ``predict`` / ``system_one`` / ``warmup`` /
  ``close`` / context management (``engine.py:216-243``);
* ``result["engine"]`` with ``graph_miss``, ``graph_build_ms``, ``shape``,
  ``backend``, ``total_ms`` (plus ``precision`` and ``device``).

The forward itself runs in liblaya_b200.so; there is no CPU path.
"""
from collections import OrderedDict
import ctypes
import queue
import threading
import time

import numpy as np

from . import _lib
from .config import LAYA, LayaConfig
from .protocol import PreparedRequest, format_response, prepare_request
from .weights import check_weights, seeded_weights, param_table
from .workload import pack

KEYS = ("input_ids", "attention_mask", "marker_pos", "marker_mask", "qtype")


def _device_index(device):
    if isinstance(device, int):
        return device
    text = str(device)
    if text == "cuda":
        return 0
    if text.startswith("cuda:"):
        return int(text.split(":", 1)[1])
    raise RuntimeError(f"the b200 mode runs on CUDA devices only; got {device!r}")


class NativeForward:
    """One engine of liblaya_b200.so on one GPU (weights, graphs, pinned I/O)."""

    def __init__(self, device, cfg: LayaConfig, weights, precision="bf16", max_batch=64, max_options=256):
        if precision not in _lib.PRECISIONS:
            raise ValueError("precision must be bf16, fp8 or nvfp4")
        cfg.validate()
        check_weights(weights, cfg)
        self.lib = _lib.load()
        self.cfg = cfg
        self.precision = precision
        self.device = device
        self.max_batch, self.max_options = max_batch, max_options
        handle = ctypes.c_void_p()
        c = _lib.make_config(cfg, max_batch, max_options)
        if self.lib.laya_b200_create(device, ctypes.byref(c), ctypes.byref(handle)) != 0:
            msg = self.lib.laya_b200_last_error(None)
            raise RuntimeError(f"laya_b200_create: {msg.decode() if msg else 'unknown error'}")
        self.handle = handle
        try:
            for name, _, _, _ in param_table(cfg):
                arr = np.ascontiguousarray(weights[name])
                st = self.lib.laya_b200_set_weight(self.handle, name.encode(), arr.ctypes.data, arr.nbytes)
                _lib.check(self.lib, self.handle, st, f"set_weight({name})")
            _lib.check(self.lib, self.handle,
                       self.lib.laya_b200_finalize(self.handle, _lib.PRECISIONS[precision]), "finalize")
        except Exception:
            self.close()
            raise

    def capture(self, batch, seq, options, unmasked):
        slot = ctypes.c_int()
        st = self.lib.laya_b200_capture(self.handle, batch, seq, options, int(bool(unmasked)), ctypes.byref(slot))
        _lib.check(self.lib, self.handle, st, f"capture({batch},{seq},{options})")
        return slot.value

    def release(self, slot):
        _lib.check(self.lib, self.handle, self.lib.laya_b200_release(self.handle, slot), "release")

    def run(self, slot, inputs):
        b, s = inputs["input_ids"].shape
        k = inputs["marker_pos"].shape[1]
        ids = np.ascontiguousarray(inputs["input_ids"], dtype=np.int64)
        am = np.ascontiguousarray(inputs["attention_mask"], dtype=np.int64)
        mp = np.ascontiguousarray(inputs["marker_pos"], dtype=np.int64)
        mm = np.ascontiguousarray(inputs["marker_mask"], dtype=np.uint8)
        qt = np.ascontiguousarray(inputs["qtype"], dtype=np.int64)
        logits = np.empty((b, k), dtype=np.float32)
        act = np.empty((b, 2), dtype=np.float32)
        self.run_addresses(slot, tuple(a.ctypes.data for a in (ids, am, mp, mm, qt, logits, act)))
        return logits, act

    def run_addresses(self, slot, addresses):
        """run() on host arrays given by address (ids, mask, marker_pos,
        marker_mask, qtype, logits, act), for callers that keep them."""
        _lib.check(self.lib, self.handle, self.lib.laya_b200_run(self.handle, slot, *addresses), "run")

    def replay_device(self, slot, iterations, kernel_mask=15):
        """Per-replay device milliseconds of `iterations` back-to-back replays."""
        ms = np.empty(iterations, dtype=np.float32)
        st = self.lib.laya_b200_replay_device(self.handle, slot, iterations, kernel_mask,
                                              ms.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
        _lib.check(self.lib, self.handle, st, "replay_device")
        return ms

    def kernel_count(self, slot):
        n = ctypes.c_int()
        _lib.check(self.lib, self.handle, self.lib.laya_b200_kernel_count(self.handle, slot, ctypes.byref(n)),
                   "kernel_count")
        return n.value

    def read_buffer(self, name, shape, dtype):
        """Copy the leading elements of a named activation buffer (test hook)."""
        out = np.empty(shape, dtype=dtype)
        st = self.lib.laya_b200_read_buffer(self.handle, name.encode(), out.ctypes.data, out.nbytes)
        _lib.check(self.lib, self.handle, st, f"read_buffer({name})")
        return out

    def test_withhold_stage(self, wait_limit_us=1000):
        """Test hook (failure detection): the next run() enqueues its forward
        without a graph and its first generic projection never loads its first
        pipeline stage, so that launch's bounded waits (limited to
        `wait_limit_us`) run out and the run raises RuntimeError."""
        _lib.check(self.lib, self.handle, self.lib.laya_b200_test_withhold_stage(self.handle, int(wait_limit_us)),
                   "test_withhold_stage")

    def build_token_tables(self):
        """Embedding-norm and layer-0 QKV rows of every token id on the device
        (slots captured afterwards start with one gather)."""
        _lib.check(self.lib, self.handle, self.lib.laya_b200_build_token_tables(self.handle), "build_token_tables")

    def lane(self):
        """A serving lane: another handle on the same GPU sharing these
        weights, with its own stream, activations and graphs."""
        handle = ctypes.c_void_p()
        if self.lib.laya_b200_create_lane(self.handle, ctypes.byref(handle)) != 0:
            msg = self.lib.laya_b200_last_error(None)
            raise RuntimeError(f"laya_b200_create_lane: {msg.decode() if msg else 'unknown error'}")
        other = NativeForward.__new__(NativeForward)
        other.lib, other.cfg, other.precision, other.device = self.lib, self.cfg, self.precision, self.device
        other.max_batch, other.max_options = self.max_batch, self.max_options
        other.handle = handle
        return other

    def close(self):
        if getattr(self, "handle", None):
            self.lib.laya_b200_destroy(self.handle)
            self.handle = None


class _Lane:
    """Per-lane state of a B200Engine beyond lane 0 (which is the engine's own
    native / graphs / _io)."""

    def __init__(self, native):
        self.native = native
        self.graphs = OrderedDict()
        self._io = {}


class B200Engine:
    """The ``mode="b200"`` engine: same public contract as BlackwellEngine."""

    def __init__(self, model=None, *, weights=None, config: LayaConfig = LAYA, seed=0, device="cuda:0",
                 max_graphs=8, max_questions=64, sequence_buckets=(64, 128, 256, 384, 512, 768, 1024),
                 precision="bf16", max_options=256, tokenizer=None, agent_cfg=None, temperature=None,
                 temperature_by_options=None, lanes=1, token_tables=False):
        if max_graphs < 1 or max_questions < 1:
            raise ValueError("max_graphs and max_questions must be positive")
        if lanes < 1:
            raise ValueError("lanes must be positive")
        if precision not in _lib.PRECISIONS:
            raise ValueError("precision must be bf16, fp8 or nvfp4")
        self.device = _device_index(device)
        self.lock = threading.RLock()
        self.max_graphs, self.max_questions = max_graphs, max_questions
        self.sequence_buckets = tuple(sorted(set(sequence_buckets)))
        self.precision = precision
        self.backend = f"b200-{precision}"
        self.config = config
        self.cfg = dict(agent_cfg or {"max_len": config.max_len})
        self.tokenizer = tokenizer
        self.pad_token_id = config.pad_token_id
        self.temperature = temperature
        self.temperature_by_options = temperature_by_options or {}
        self.graphs = OrderedDict()
        self.closed = False
        if weights is None:
            weights = _load_weights(model) if model is not None else seeded_weights(config, seed)
        max_options = max(2, 1 << (max_options - 1).bit_length())
        self.native = NativeForward(self.device, config, weights, precision, max_batch=max_questions,
                                    max_options=max_options)
        self.max_options = max_options
        if token_tables:  # before the lanes, which share them
            try:
                self.native.build_token_tables()
            except Exception:
                self.native.close()
                raise
        # Serving lanes: requests from concurrent callers run on idle lanes
        # (lane 0 is this object's own native / graphs); one lane serialises
        # every call like the reference's engine lock (engine.py:84,192).
        self._idle = queue.Queue()
        self._lanes = [self]
        try:
            for _ in range(lanes - 1):
                self._lanes.append(_Lane(self.native.lane()))
        except Exception:
            for lane in self._lanes[1:]:
                lane.native.close()
            self.native.close()
            raise
        for lane in self._lanes:
            self._idle.put(lane)

    # -- request preparation (needs the Laya SDK tokenizer, as the reference)
    def prepare(self, state, questions):
        if self.tokenizer is None:
            raise RuntimeError("prepare() needs the checkpoint tokenizer and the laya SDK; "
                               "pass pre-tokenized PreparedRequest objects to run_prepared()")
        from laya.common import serialize_state  # noqa: PLC0415 - optional SDK
        return prepare_request(self.tokenizer, self.cfg, serialize_state(state), questions,
                               max_questions=self.max_questions, truncate_left=isinstance(state, list))

    # -- shapes (engine.py:112-138)
    def _shape(self, prepared):
        count = len(prepared.items)
        length, options = 0, 2
        for x in prepared.items:
            n, k = len(x["ids"]), len(x["markers"])
            if n > length:
                length = n
            if k > options:
                options = k
        max_len = self.cfg.get("max_len", 512)
        length = next((x for x in self.sequence_buckets if length <= x <= max_len), max_len)
        batch = min(self.max_questions, 1 << (count - 1).bit_length())
        return batch, length, 1 << (options - 1).bit_length()

    def _graph_key(self, prepared):
        shape = self._shape(prepared)
        batch, length, _ = shape
        unmasked = len(prepared.items) == batch and all(len(item["ids"]) == length for item in prepared.items)
        return (*shape, unmasked)

    def _fill(self, prepared, shape):
        batch, length, options = shape
        return pack(prepared.items, batch, length, options, self.pad_token_id)

    def _run_slot(self, slot, key, prepared, lane=None):
        """Pack into the slot's own host arrays (kept per graph key, addresses
        computed once) and run; same values as _fill + NativeForward.run."""
        lane = lane or self
        if not hasattr(lane.native, "run_addresses"):
            return lane.native.run(slot, self._fill(prepared, key[:3]))
        io = getattr(lane, "_io", None)
        if io is None:
            io = lane._io = {}
        bufs = io.get(key)
        if bufs is None:
            batch, length, options = key[:3]
            # the int64 inputs are views of one block, reset from a pristine
            # copy (pad ids, dummy rows seeing their position 0) in one copy
            cuts = np.cumsum([batch * length, batch * length, batch * options, batch])
            ints = np.empty(int(cuts[-1]), np.int64)
            ids, mask, mpos, qtype = np.split(ints, cuts[:-1])
            arrays = {"input_ids": ids.reshape(batch, length),
                      "attention_mask": mask.reshape(batch, length),
                      "marker_pos": mpos.reshape(batch, options),
                      "marker_mask": np.empty((batch, options), np.uint8),
                      "qtype": qtype,
                      "logits": np.empty((batch, options), np.float32),
                      "act": np.empty((batch, 2), np.float32)}
            clean_ints = np.zeros_like(ints)
            clean_ints[:batch * length] = self.pad_token_id
            clean_ints[batch * length:2 * batch * length].reshape(batch, length)[:, 0] = 1
            clean_mmask = np.zeros((batch, options), np.uint8)
            clean_mmask[:, 0] = 1
            bufs = io[key] = (arrays, tuple(a.ctypes.data for a in arrays.values()), ints, clean_ints,
                              clean_mmask)
        arrays, addresses, ints, clean_ints, clean_mmask = bufs
        ids, mask, mpos, mmask, qtype = (arrays[n] for n in ("input_ids", "attention_mask", "marker_pos",
                                                             "marker_mask", "qtype"))
        np.copyto(ints, clean_ints)
        np.copyto(mmask, clean_mmask)
        for i, item in enumerate(prepared.items):
            n, k = len(item["ids"]), len(item["markers"])
            ids[i, :n] = item["ids"]
            mask[i, :n] = 1
            mpos[i, :k] = item["markers"]
            mmask[i, :k] = 1
            qtype[i] = item["qtype"]
        lane.native.run_addresses(slot, addresses)
        return arrays["logits"], arrays["act"]

    def _check_items(self, prepared, shape):
        _, length, options = shape
        for item in prepared.items:
            if len(item["ids"]) > length:
                raise ValueError(f"question has {len(item['ids'])} tokens; the model maximum is {length}")
            if len(item["markers"]) > options or len(item["markers"]) > self.max_options:
                raise ValueError(f"question has {len(item['markers'])} options; maximum is {self.max_options}")

    def _slot(self, prepared, key=None, lane=None):
        lane = lane or self
        key = key or self._graph_key(prepared)
        if key in lane.graphs:
            lane.graphs.move_to_end(key)
            return lane.graphs[key], False, 0.0
        if len(lane.graphs) >= self.max_graphs:
            old_key, old = lane.graphs.popitem(last=False)
            lane.native.release(old)
            getattr(lane, "_io", {}).pop(old_key, None)
        start = time.perf_counter()
        slot = lane.native.capture(*key)
        lane.graphs[key] = slot
        return slot, True, (time.perf_counter() - start) * 1000

    def run_prepared(self, prepared):
        """Returns owned CPU arrays (logits [n, k_padded], act [n, 2], metrics)."""
        idle = getattr(self, "_idle", None)
        if idle is None:  # engines assembled without lanes
            with self.lock:
                if self.closed:
                    raise RuntimeError("Engine is closed")
                return self._run_on(prepared, self)
        lane = idle.get()
        try:
            if self.closed:
                raise RuntimeError("Engine is closed")
            return self._run_on(prepared, lane)
        finally:
            idle.put(lane)

    def _run_on(self, prepared, lane):
        if not prepared.items:
            return np.empty((0, 0)), np.empty((0, 2)), {"graph_miss": False}
        key = self._graph_key(prepared)
        shape = key[:3]
        self._check_items(prepared, shape)
        slot, miss, build_ms = self._slot(prepared, key, lane)
        logits, act = self._run_slot(slot, key, prepared, lane)
        count = len(prepared.items)
        return logits[:count].copy(), act[:count].copy(), {
            "graph_miss": miss, "graph_build_ms": build_ms if miss else 0.0, "shape": list(shape),
            "backend": self.backend, "precision": self.precision, "device": f"cuda:{self.device}"}

    def predict(self, state, questions):
        start = time.perf_counter()
        prepared = self.prepare(state, questions)
        logits, act, metrics = self.run_prepared(prepared)
        result = format_response(prepared, logits, act, self.temperature, self.temperature_by_options)
        metrics["total_ms"] = (time.perf_counter() - start) * 1000
        result["engine"] = metrics
        return result

    system_one = predict

    def warmup(self, state, questions):
        return self.predict(state, questions)["engine"]

    def close(self):
        with self.lock:
            if self.closed:
                return
            lanes = getattr(self, "_lanes", [self])
            idle = getattr(self, "_idle", None)
            if idle is not None:  # wait for every lane to be idle
                held = [idle.get() for _ in lanes]
            self.closed = True
            for lane in lanes:
                lane.graphs.clear()
                getattr(lane, "_io", {}).clear()
            for lane in lanes[1:]:  # lanes before the weights' owner
                lane.native.close()
            if getattr(self, "native", None) is not None:
                self.native.close()
            self.native = None
            if idle is not None:
                for lane in held:
                    idle.put(lane)

    def __enter__(self):
        return self

    def __exit__(self, *_):
        self.close()


def _load_weights(path):
    """Weights from an .npz holding the parameter table (bf16 as uint16)."""
    with np.load(path) as z:
        return {k: z[k] for k in z.files}


def request_from_items(items):
    """A PreparedRequest for already-tokenised items (ids, markers, qtype)."""
    return PreparedRequest([str(i) for i in range(len(items))], [{} for _ in items], list(items),
                           sum(len(it["ids"]) for it in items))
