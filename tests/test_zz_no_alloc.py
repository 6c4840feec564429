"""The allocation-free decision tail (laya_b200_tail_noalloc) against the
engine's own tail inside laya_b200_run.

This entry point exists for callers that cannot allocate device memory
(a host that owns every device buffer through its own allocator or pool, or a
worker limited to launching on memory it was handed).  The test runs a full
forward through laya_b200_run, reads the tail's inputs back, hands them to the
allocation-free entry point as caller-owned device buffers and checks that two
calls in a row reproduce the engine's logits and act within the bf16 forward
tolerance (2e-2 max-abs).  It is collected last so that a failure here cannot
hide the other tests' results, and it passes alone in a fresh process too.
"""
import ctypes

import numpy as np
import pytest

from laya_b200.config import TINY
from laya_b200.weights import seeded_weights
from laya_b200.workload import synthetic_items, pack

pytestmark = pytest.mark.gpu

TOL = 2e-2


def test_tail_noalloc_matches_engine_tail():
    import torch
    from laya_b200 import _lib
    from laya_b200.engine import NativeForward

    cfg = TINY
    w = seeded_weights(cfg, seed=7)
    b, s, k = 4, 96, 4
    items = synthetic_items([96, 50, 20], ["choice", "score", "noul"], seed=9, vocab=cfg.vocab)
    inp = pack(items, b, s, k, cfg.pad_token_id)
    nf = NativeForward(0, cfg, w, "bf16", max_batch=b, max_options=k)
    try:
        slot = nf.capture(b, s, k, False)
        ref_logits, ref_act = nf.run(slot, inp)
        z = nf.read_buffer("zsc", (b * k, cfg.hidden), np.uint16)
        hsel = nf.read_buffer("hsel", (b * (1 + k), cfg.hidden), np.float32)
    finally:
        nf.close()

    dev = torch.device("cuda", 0)

    def up(a, dtype):
        return torch.from_numpy(np.ascontiguousarray(a).view(dtype)).to(dev)

    bufs = {
        "z": up(z, np.int16), "fc2_w": up(w["scorer.fc2.w"], np.int16), "fc2_b": up(w["scorer.fc2.b"], np.int16),
        "marker_mask": up(inp["marker_mask"].astype(np.int32), np.int32), "h_sel": up(hsel, np.float32),
        "a1_w": up(w["act.fc1.w"], np.int16), "a1_b": up(w["act.fc1.b"], np.int16),
        "a2_w": up(w["act.fc2.w"], np.int16), "a2_b": up(w["act.fc2.b"], np.int16),
    }
    logits = torch.empty((b, k), dtype=torch.float32, device=dev)
    act = torch.empty((b, 2), dtype=torch.float32, device=dev)
    args = _lib.TailArgs(questions=b, options=k, hidden=cfg.hidden, act_hidden=cfg.act_hidden,
                         logits=logits.data_ptr(), act=act.data_ptr(),
                         **{name: t.data_ptr() for name, t in bufs.items()})
    lib = _lib.load()
    stream = torch.cuda.current_stream(dev)
    for call in range(2):
        logits.fill_(float("nan"))
        act.fill_(float("nan"))
        st = lib.laya_b200_tail_noalloc(ctypes.byref(args), ctypes.c_void_p(stream.cuda_stream))
        assert st == 0, lib.laya_b200_last_error(None)
        torch.cuda.synchronize(dev)
        got_l, got_a = logits.cpu().numpy(), act.cpu().numpy()
        assert np.isfinite(got_l).all() and np.isfinite(got_a).all(), call
        assert np.abs(got_l - ref_logits).max() <= TOL, (call, got_l, ref_logits)
        assert np.abs(got_a - ref_act).max() <= TOL, (call, got_a, ref_act)


def test_tail_noalloc_rejects_oversized_calls():
    from laya_b200 import _lib
    lib = _lib.load()
    args = _lib.TailArgs(questions=65, options=4, hidden=256, act_hidden=64)
    assert lib.laya_b200_tail_noalloc(ctypes.byref(args), None) != 0
    assert b"questions" in lib.laya_b200_last_error(None)
    args = _lib.TailArgs(questions=64, options=4, hidden=256, act_hidden=1025)
    assert lib.laya_b200_tail_noalloc(ctypes.byref(args), None) != 0
