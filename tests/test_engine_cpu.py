"""B200Engine shape, graph-key, fill and lifetime semantics without CUDA,
mirroring the reference's tests/test_engine_cpu.py tables."""
from collections import OrderedDict
import threading

import numpy as np
import pytest

from laya_b200.config import TINY
from laya_b200.engine import B200Engine, request_from_items, _device_index
from laya_b200.protocol import PreparedRequest
from laya_b200.workload import pack, synthetic_items


class FakeNative:
    def __init__(self):
        self.captured, self.released, self.runs = [], [], 0
        self.closed = False

    def capture(self, b, s, k, unmasked):
        self.captured.append((b, s, k, unmasked))
        return len(self.captured) - 1

    def release(self, slot):
        self.released.append(slot)

    def run(self, slot, inputs):
        self.runs += 1
        b, k = inputs["marker_pos"].shape
        return np.full((b, k), float(slot), np.float32), np.zeros((b, 2), np.float32)

    def close(self):
        self.closed = True


def make_engine(*, max_questions=64, max_len=512, max_graphs=8):
    engine = B200Engine.__new__(B200Engine)
    engine.lock = threading.RLock()
    engine.max_questions, engine.max_graphs = max_questions, max_graphs
    engine.sequence_buckets = (64, 128, 256, 384, 512, 768, 1024)
    engine.cfg = {"max_len": max_len}
    engine.pad_token_id = 0
    engine.max_options = 256
    engine.backend, engine.precision, engine.device = "b200-bf16", "bf16", 0
    engine.graphs = OrderedDict()
    engine.closed = False
    engine.native = FakeNative()
    return engine


def request_with_shapes(*shapes):
    items = [{"ids": [10] * length, "markers": list(range(options)), "qtype": index % 3}
             for index, (length, options) in enumerate(shapes)]
    return PreparedRequest([str(i) for i in range(len(items))], [{}] * len(items), items,
                           sum(len(item["ids"]) for item in items))


@pytest.mark.parametrize("shapes, limit, max_len, expected", [
    ([(1, 1)], 64, 512, (1, 64, 2)),
    ([(65, 3)], 64, 512, (1, 128, 4)),
    ([(65, 3), (80, 2), (20, 1)], 64, 512, (4, 128, 4)),
    ([(20, 2)] * 5, 6, 512, (6, 64, 2)),
    ([(80, 2)], 64, 96, (1, 96, 2)),
    ([(512, 65)], 64, 512, (1, 512, 128)),
])
def test_shape_buckets_match_reference_table(shapes, limit, max_len, expected):
    engine = make_engine(max_questions=limit, max_len=max_len)
    assert engine._shape(request_with_shapes(*shapes)) == expected


@pytest.mark.parametrize("shapes, unmasked", [
    ([(64, 2)], True), ([(63, 2)], False), ([(64, 2), (64, 2)], True),
    ([(64, 2), (63, 2)], False), ([(64, 2)] * 3, False),
])
def test_graph_key_separates_unmasked(shapes, unmasked):
    engine = make_engine()
    prepared = request_with_shapes(*shapes)
    assert engine._graph_key(prepared) == (*engine._shape(prepared), unmasked)


def test_fill_pads_dummy_rows_like_the_reference():
    prepared = request_with_shapes((3, 2), (2, 1))
    prepared.items[0]["ids"] = [1, 3, 2]
    prepared.items[1]["ids"] = [1, 2]
    buf = pack(prepared.items, 4, 8, 4, 0)
    assert buf["input_ids"].tolist() == [[1, 3, 2, 0, 0, 0, 0, 0], [1, 2, 0, 0, 0, 0, 0, 0], [0] * 8, [0] * 8]
    assert buf["attention_mask"].tolist() == [[1, 1, 1, 0, 0, 0, 0, 0], [1, 1, 0, 0, 0, 0, 0, 0],
                                              [1, 0, 0, 0, 0, 0, 0, 0], [1, 0, 0, 0, 0, 0, 0, 0]]
    assert buf["marker_pos"].tolist() == [[0, 1, 0, 0], [0] * 4, [0] * 4, [0] * 4]
    assert buf["marker_mask"].tolist() == [[True, True, False, False], [True, False, False, False],
                                           [True, False, False, False], [True, False, False, False]]
    assert buf["qtype"].tolist() == [0, 1, 0, 0]


def test_closed_engine_rejects_requests():
    engine = make_engine()
    engine.closed = True
    with pytest.raises(RuntimeError, match="Engine is closed"):
        engine.run_prepared(request_with_shapes())


def test_empty_request_creates_no_graph():
    engine = make_engine()
    logits, act, metrics = engine.run_prepared(request_with_shapes())
    assert logits.shape == (0, 0) and act.shape == (0, 2) and metrics["graph_miss"] is False
    assert not engine.graphs and not engine.native.captured


def test_graph_cache_hits_and_lru_eviction_release_slots():
    engine = make_engine(max_graphs=2)
    a, b, c = request_with_shapes((64, 2)), request_with_shapes((100, 2)), request_with_shapes((300, 4))
    assert engine.run_prepared(a)[2]["graph_miss"] is True
    assert engine.run_prepared(a)[2]["graph_miss"] is False
    engine.run_prepared(b)
    engine.run_prepared(c)           # evicts a's slot
    assert engine.native.released == [0]
    assert list(engine.graphs) == [(1, 128, 2, False), (1, 384, 4, False)]
    assert engine.run_prepared(a)[2]["graph_miss"] is True


def test_outputs_are_owned_copies_and_metrics_have_reference_keys():
    engine = make_engine()
    logits, act, metrics = engine.run_prepared(request_with_shapes((64, 2), (10, 2), (5, 2)))
    assert logits.shape == (3, 2) and act.shape == (3, 2)
    assert logits.base is None or logits.base is not engine.native
    assert {"graph_miss", "graph_build_ms", "shape", "backend"} <= set(metrics)
    assert metrics["shape"] == [4, 64, 2]


def test_oversized_questions_are_rejected_before_device_work():
    engine = make_engine(max_len=96)
    with pytest.raises(ValueError, match="tokens"):
        engine.run_prepared(request_with_shapes((97, 2)))
    assert engine.native.runs == 0


def test_close_is_idempotent_and_releases_native():
    engine = make_engine()
    native = engine.native
    engine.close()
    engine.close()
    assert native.closed and engine.closed and engine.native is None


def test_constructor_validation_happens_before_native_work():
    with pytest.raises(ValueError, match="positive"):
        B200Engine(max_graphs=0)
    with pytest.raises(ValueError, match="precision"):
        B200Engine(precision="int4")
    with pytest.raises(RuntimeError, match="CUDA devices only"):
        _device_index("cpu")


def test_request_from_items_counts_tokens():
    items = [{"ids": [1, 2, 3], "markers": [1, 2], "qtype": 0}, {"ids": [4], "markers": [0, 0], "qtype": 2}]
    req = request_from_items(items)
    assert req.input_tokens == 4 and len(req.ids) == 2


class AddressNative(FakeNative):
    """A native stand-in that reads run()'s host arrays back from their
    addresses, as the C ABI does."""

    def __init__(self):
        super().__init__()
        self.seen = []

    def run_addresses(self, slot, addresses):
        import ctypes
        b, s, k = self.captured[slot][:3]
        def view(addr, shape, dtype):
            n = int(np.prod(shape)) * np.dtype(dtype).itemsize
            return np.frombuffer((ctypes.c_char * n).from_address(addr), dtype=dtype).reshape(shape).copy()
        ids, mask, mpos, mmask, qtype = (view(addresses[0], (b, s), np.int64), view(addresses[1], (b, s), np.int64),
                                         view(addresses[2], (b, k), np.int64), view(addresses[3], (b, k), np.uint8),
                                         view(addresses[4], (b,), np.int64))
        self.seen.append({"input_ids": ids, "attention_mask": mask, "marker_pos": mpos,
                          "marker_mask": mmask.astype(bool), "qtype": qtype})
        logits = np.frombuffer((ctypes.c_char * (b * k * 4)).from_address(addresses[5]), np.float32)
        logits[:] = float(slot)


def test_run_packs_into_kept_host_arrays_like_fill():
    """run_prepared's in-place packing into per-slot host arrays gives the
    arrays _fill builds (BlackwellEngine._fill semantics), across calls that
    reuse the arrays with fewer questions and shorter rows."""
    engine = make_engine(max_questions=4)
    engine.native = AddressNative()
    first = synthetic_items([64, 40, 12], ["choice", "noul", "score"], seed=4, vocab=1000)
    second = synthetic_items([30, 20], ["noul", "noul"], seed=5, vocab=1000)
    # same graph key as `first`, other row lengths and options: every stale
    # value of the previous call must be reset
    third = synthetic_items([12, 64, 7], ["score", "choice", "noul"], seed=6, vocab=1000)
    for items in (first, second, first, third):
        prepared = request_from_items(items)
        engine.run_prepared(prepared)
        shape = engine._shape(prepared)
        want = engine._fill(prepared, shape)
        got = engine.native.seen[-1]
        for name in want:
            assert np.array_equal(got[name], want[name]), name


def test_lanes_serve_concurrent_callers():
    """With two lanes, two callers run at the same time, each on its own lane
    (own native handle and graph slots); a third caller waits for an idle lane;
    close() waits for the lanes and later calls raise."""
    import queue
    from laya_b200.engine import _Lane

    class SlowNative(FakeNative):
        def __init__(self, gate):
            super().__init__()
            self.gate = gate

        def run(self, slot, inputs):
            self.gate.wait(5)
            return super().run(slot, inputs)

    gate = threading.Event()
    engine = make_engine(max_questions=4)
    engine.native = SlowNative(gate)
    engine._lanes = [engine, _Lane(SlowNative(gate))]
    engine._idle = queue.Queue()
    for lane in engine._lanes:
        engine._idle.put(lane)
    prepared = request_from_items(synthetic_items([30], ["noul"], seed=2, vocab=1000))
    results = []
    threads = [threading.Thread(target=lambda: results.append(engine.run_prepared(prepared))) for _ in range(3)]
    for t in threads:
        t.start()
    import time
    time.sleep(0.2)
    assert engine._idle.qsize() == 0          # both lanes busy, the third caller waits
    gate.set()
    for t in threads:
        t.join(5)
    assert len(results) == 3
    assert engine.native.runs + engine._lanes[1].native.runs == 3
    assert engine.native.runs >= 1 and engine._lanes[1].native.runs >= 1
    assert engine.graphs and engine._lanes[1].graphs  # each lane captured its own slot
    engine.close()
    with pytest.raises(RuntimeError, match="closed"):
        engine.run_prepared(prepared)


def test_predict_warmup_and_system_one_follow_the_reference_contract(monkeypatch):
    """predict = prepare -> run_prepared -> format_response, with the engine
    metrics under result["engine"] and total_ms added last; system_one is
    predict and warmup returns the metrics alone (engine.py:216-229 of the
    reference).  The Laya SDK and the reference protocol are faked: prepare()
    must serialise the state with laya.common.serialize_state, tokenise with
    the engine's tokenizer and config, and truncate left for list states."""
    import sys
    import types
    from laya_b200 import engine as engine_module

    calls = []
    common = types.ModuleType("laya.common")
    common.serialize_state = lambda state: ("serialized", tuple(state) if isinstance(state, list) else state)
    sdk = types.ModuleType("laya")
    sdk.common = common
    monkeypatch.setitem(sys.modules, "laya", sdk)
    monkeypatch.setitem(sys.modules, "laya.common", common)

    def fake_prepare(tok, cfg, state, questions, **kwargs):
        calls.append(("prepare", tok, dict(cfg), state, len(questions), kwargs))
        items = [{"ids": [7] * (20 + 10 * i), "markers": [1, 2, 3][: 2 + i % 2], "qtype": i % 3}
                 for i in range(len(questions))]
        return PreparedRequest([q["id"] for q in questions], list(questions), items,
                               sum(len(it["ids"]) for it in items))

    def fake_format(prepared, logits, act, temperature, temperature_by_options):
        calls.append(("format", logits.shape, act.shape, temperature, dict(temperature_by_options)))
        return {"answers": {qid: int(np.argmax(logits[i])) for i, qid in enumerate(prepared.ids)}}

    monkeypatch.setattr(engine_module, "prepare_request", fake_prepare)
    monkeypatch.setattr(engine_module, "format_response", fake_format)
    engine = make_engine(max_questions=4)
    engine.tokenizer = "tok"
    engine.temperature, engine.temperature_by_options = 1.5, {2: 0.5}
    questions = [{"id": "q0"}, {"id": "q1"}, {"id": "q2"}]

    result = engine.predict(["a", "b"], questions)
    assert set(result) == {"answers", "engine"}
    assert set(result["answers"]) == {"q0", "q1", "q2"}
    metrics = result["engine"]
    assert {"graph_miss", "graph_build_ms", "shape", "backend", "total_ms"} <= set(metrics)
    assert metrics["graph_miss"] is True and metrics["shape"] == [4, 64, 4]
    assert metrics["backend"] == "b200-bf16" and metrics["total_ms"] >= 0.0
    assert list(metrics)[-1] == "total_ms"
    kind, tok, cfg, state, count, kwargs = calls[0]
    assert (kind, tok, cfg, count) == ("prepare", "tok", {"max_len": 512}, 3)
    assert state == ("serialized", ("a", "b"))
    assert kwargs == {"max_questions": 4, "truncate_left": True}
    assert calls[1] == ("format", (3, 4), (3, 2), 1.5, {2: 0.5})

    # system_one is predict; the same shape now hits the captured graph
    again = engine.system_one({"k": 1}, questions)
    assert again["engine"]["graph_miss"] is False and again["engine"]["graph_build_ms"] == 0.0
    assert calls[2][3] == ("serialized", {"k": 1}) and calls[2][5]["truncate_left"] is False

    # warmup returns the metrics dictionary only, total_ms included
    warm = engine.warmup({"k": 1}, questions[:1])
    assert set(warm) >= {"graph_miss", "shape", "total_ms"} and warm["shape"] == [1, 64, 2]
    assert engine.native.captured == [(4, 64, 4, False), (1, 64, 2, False)]


def test_prepare_without_tokenizer_names_what_is_missing():
    engine = make_engine()
    engine.tokenizer = None
    with pytest.raises(RuntimeError, match="tokenizer"):
        engine.predict({}, [{"id": "q"}])


@pytest.mark.parametrize("changes, message", [
    ({"max_len": 768}, "max_len"),      # attention keeps a query's 512 scores in tensor memory
    ({"max_len": 0}, "max_len"),
    ({"head_dim": 32}, "head dimension"),
])
def test_config_validation_names_the_limit(changes, message):
    from dataclasses import replace
    from laya_b200.config import LAYA
    with pytest.raises(ValueError, match=message):
        replace(LAYA, **changes).validate()
    LAYA.validate()
