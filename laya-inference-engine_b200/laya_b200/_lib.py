"""ctypes binding of liblaya_b200.so (the C ABI in include/laya_b200.h).

The library is built in-tree by ``laya-inference-engine_b200/build.py``.  There
is no fallback: if it is missing or fails to load, every engine constructor
raises.  ctypes releases the GIL for the duration of each foreign call, so one
thread per GPU can drive its engine concurrently.
"""
import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().with_name("liblaya_b200.so")

PRECISIONS = {"bf16": 0, "fp8": 1, "nvfp4": 2}

EXPORTS = ("laya_b200_create", "laya_b200_set_weight", "laya_b200_finalize", "laya_b200_create_lane",
           "laya_b200_build_token_tables",
           "laya_b200_capture",
           "laya_b200_release", "laya_b200_run", "laya_b200_replay_device", "laya_b200_kernel_count",
           "laya_b200_read_buffer", "laya_b200_tail_noalloc", "laya_b200_test_withhold_stage",
           "laya_b200_last_error", "laya_b200_destroy")


class Config(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in ("layers", "hidden", "heads", "head_dim", "intermediate", "vocab",
                                                "max_len", "local_window", "global_every")] + \
               [(n, ctypes.c_float) for n in ("rope_theta_global", "rope_theta_local", "norm_eps")] + \
               [(n, ctypes.c_int32) for n in ("head_layers", "head_heads", "head_ff", "num_qtypes", "act_hidden",
                                                "max_batch", "max_options")]


class TailArgs(ctypes.Structure):
    """laya_b200_tail_args: device pointers owned by the caller."""
    _fields_ = [(n, ctypes.c_int32) for n in ("questions", "options", "hidden", "act_hidden")] + \
               [(n, ctypes.c_void_p) for n in ("z", "fc2_w", "fc2_b", "marker_mask", "h_sel", "a1_w", "a1_b",
                                                "a2_w", "a2_b", "logits", "act")]


def make_config(cfg, max_batch, max_options):
    return Config(layers=cfg.layers, hidden=cfg.hidden, heads=cfg.heads, head_dim=cfg.head_dim,
                  intermediate=cfg.intermediate, vocab=cfg.vocab, max_len=cfg.max_len,
                  local_window=cfg.window, global_every=cfg.global_every,
                  rope_theta_global=cfg.rope_theta_global, rope_theta_local=cfg.rope_theta_local,
                  norm_eps=cfg.norm_eps, head_layers=cfg.head_layers, head_heads=cfg.head_heads,
                  head_ff=cfg.head_ff, num_qtypes=cfg.num_qtypes, act_hidden=cfg.act_hidden,
                  max_batch=max_batch, max_options=max_options)


_LIB = None


def load():
    """Load the shared library once; raise RuntimeError when it is absent."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not LIB_PATH.exists():
        raise RuntimeError(f"{LIB_PATH.name} is not built; run `python laya-inference-engine_b200/build.py` "
                           "(the b200 mode has no CPU fallback)")
    lib = ctypes.CDLL(str(LIB_PATH))
    P, I, F = ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(ctypes.c_float)
    sig = {
        "laya_b200_create": (I, [I, ctypes.POINTER(Config), ctypes.POINTER(P)]),
        "laya_b200_create_lane": (I, [P, ctypes.POINTER(P)]),
        "laya_b200_build_token_tables": (I, [P]),
        "laya_b200_set_weight": (I, [P, ctypes.c_char_p, P, ctypes.c_size_t]),
        "laya_b200_finalize": (I, [P, I]),
        "laya_b200_capture": (I, [P, I, I, I, I, ctypes.POINTER(I)]),
        "laya_b200_release": (I, [P, I]),
        # host arrays by address (int64 ids / mask / marker_pos / qtype, uint8
        # marker_mask, fp32 logits / act)
        "laya_b200_run": (I, [P, I, P, P, P, P, P, P, P]),
        "laya_b200_replay_device": (I, [P, I, I, I, F]),
        "laya_b200_kernel_count": (I, [P, I, ctypes.POINTER(I)]),
        "laya_b200_read_buffer": (I, [P, ctypes.c_char_p, P, ctypes.c_size_t]),
        "laya_b200_tail_noalloc": (I, [ctypes.POINTER(TailArgs), P]),
        "laya_b200_test_withhold_stage": (I, [P, I]),
        "laya_b200_last_error": (ctypes.c_char_p, [P]),
        "laya_b200_destroy": (I, [P]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype, fn.argtypes = res, args
    _LIB = lib
    return lib


def check(lib, handle, status, what):
    if status != 0:
        msg = lib.laya_b200_last_error(handle)
        raise RuntimeError(f"{what}: {msg.decode() if msg else 'unknown error'}")
