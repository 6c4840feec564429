"""The C ABI library: it loads without a GPU, exports every function that
include/laya_b200.h declares, and fails cleanly (no crash) when no GPU is
present.  No compute calls."""
import ctypes
import re
from pathlib import Path

import pytest
import torch

from laya_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "laya_b200.h"


def declared():
    return re.findall(r"LAYA_B200_API\s+[\w\s\*]+?\b(laya_b200_\w+)\s*\(", HEADER.read_text())


def test_every_declared_function_is_exported():
    names = declared()
    assert len(names) >= 10
    lib = _lib.load()
    for n in names:
        assert hasattr(lib, n), n
    assert set(names) == set(_lib.EXPORTS)


def test_destroy_null_is_safe():
    assert _lib.load().laya_b200_destroy(None) == 0


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU failure path")
def test_create_without_gpu_fails_with_message():
    from laya_b200.config import TINY
    lib = _lib.load()
    h = ctypes.c_void_p()
    cfg = _lib.make_config(TINY, 2, 4)
    assert lib.laya_b200_create(0, ctypes.byref(cfg), ctypes.byref(h)) != 0
    assert h.value is None
    assert lib.laya_b200_last_error(None)


def test_create_rejects_bad_shapes_before_touching_the_gpu():
    from laya_b200.config import TINY
    import dataclasses
    lib = _lib.load()
    h = ctypes.c_void_p()
    bad = dataclasses.replace(TINY, head_dim=32, hidden=128)
    cfg = _lib.make_config(bad, 2, 4)
    assert lib.laya_b200_create(0, ctypes.byref(cfg), ctypes.byref(h)) != 0
    assert b"head_dim" in lib.laya_b200_last_error(None)


def test_tail_noalloc_validates_before_any_cuda_call():
    lib = _lib.load()
    args = _lib.TailArgs(questions=0, options=4, hidden=256, act_hidden=64)
    assert lib.laya_b200_tail_noalloc(ctypes.byref(args), None) != 0
    assert b"questions" in lib.laya_b200_last_error(None)


def test_tail_noalloc_rejects_unaligned_vector_operands():
    """z and fc2_w are read 16 bytes at a time on the GPU; a pointer that is
    only 8-byte aligned is refused on the host before any CUDA call."""
    lib = _lib.load()
    base = 1 << 20
    good = dict(questions=2, options=4, hidden=256, act_hidden=64, fc2_b=base, marker_mask=base, h_sel=base,
                a1_w=base, a1_b=base, a2_w=base, a2_b=base, logits=base, act=base)
    for name in ("z", "fc2_w"):
        ptrs = {"z": base, "fc2_w": base, name: base + 8}
        args = _lib.TailArgs(**good, **ptrs)
        assert lib.laya_b200_tail_noalloc(ctypes.byref(args), None) != 0
        assert b"16-byte aligned" in lib.laya_b200_last_error(None)
