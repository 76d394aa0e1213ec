"""ctypes binding of the C ABI in ``include/tree_attn.h``.

The shared library is built in-tree by ``build.py`` (``libtree_attn_b200.so``
next to this file).  There is no fallback: if the library is missing or was
built for another ABI version, every kernel entry point raises.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().with_name("libtree_attn_b200.so")
ABI_VERSION = 5

DTYPE_BF16 = 1
DTYPE_F16 = 2

ERR_ARG = 1
ERR_LAUNCH = 2
ERR_BOUNDS = 4
ERR_TIMEOUT = 8
ERR_UNSUPPORTED = 16
ERR_TOO_LARGE = 32
NOALLOC_SCRATCH_BYTES = 32 << 20

STATUS_NAMES = {ERR_ARG: "invalid argument", ERR_LAUNCH: "kernel launch failed",
                ERR_BOUNDS: "plan index out of range on the device",
                ERR_TIMEOUT: "bounded device wait gave up",
                ERR_UNSUPPORTED: "shape or dtype not supported",
                ERR_TOO_LARGE: "problem exceeds a fixed scratch or buffer size"}

# Every symbol declared in include/tree_attn.h.
EXPORTS = ("ta_abi_version", "ta_error_string", "ta_segment", "ta_merge", "ta_attention",
           "ta_attention_noalloc", "ta_update_tail_klen", "ta_decode_append", "ta_plan_build", "ta_schedule_tree")

SCHEDULE_GREEDY = 1
SCHEDULE_CUBE = 2


class PlanLayout(ctypes.Structure):
    """Mirror of ``ta_plan_layout``."""
    _fields_ = [(name, ctypes.c_int32) for name in (
        "num_jobs", "max_requests", "max_slots", "num_requests", "num_pieces", "num_partials", "max_pslots",
        "num_small_tasks", "num_tc_tasks", "num_kn_tasks", "num_kn_segs", "kn_ctas")]
    _fields_ += [("kn_class_ctas", ctypes.c_int32 * 5), ("small_class_end", ctypes.c_int32 * 3)]
    _fields_ += [(name, ctypes.c_int32) for name in (
        "small_max_keys", "kstart_stride", "off_qids", "off_kstart", "off_qlen", "off_klen", "off_slots",
        "off_counts", "off_pieces", "off_pcounts", "off_cslots", "off_small_tasks", "off_tc_tasks",
        "off_kn_offsets", "off_kn_tasks", "off_kn_segs")]


class CostModelC(ctypes.Structure):
    """Mirror of ``ta_cost_model``."""
    _fields_ = [("bandwidth", ctypes.c_double), ("cube_flops", ctypes.c_double), ("task_us", ctypes.c_double),
                ("merge_us", ctypes.c_double), ("cube_rows", ctypes.c_int32), ("key_tile", ctypes.c_int32),
                ("kv_split", ctypes.c_int32), ("max_query_rows", ctypes.c_int32)]


def describe_status(code):
    if code == 0:
        return "ok"
    return ", ".join(name for bit, name in STATUS_NAMES.items() if code & bit) or f"status {code}"


_lib = None


def load():
    """Load the kernel library once; raise if it is absent or mismatched."""
    global _lib
    if _lib is not None:
        return _lib
    path = os.environ.get("TREE_ATTN_LIB", str(LIB_PATH))
    if not Path(path).exists():
        raise RuntimeError(f"tree-attention kernel library not found at {path}; "
                           "build it with `python tree-attention-scheduling_b200/build.py`")
    lib = ctypes.CDLL(path)
    P, I32, I64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64
    LP = ctypes.POINTER(PlanLayout)
    lib.ta_abi_version.restype = ctypes.c_int
    lib.ta_abi_version.argtypes = []
    lib.ta_error_string.restype = ctypes.c_char_p
    lib.ta_error_string.argtypes = [ctypes.c_int]
    lib.ta_segment.restype = ctypes.c_int
    lib.ta_segment.argtypes = [LP, P, P, P, P, I64, I32, I32, I32, I32, P, P, P, P]
    lib.ta_merge.restype = ctypes.c_int
    lib.ta_merge.argtypes = [LP, P, P, P, P, P, I32, I32, I32, I32, P, P]
    lib.ta_attention.restype = ctypes.c_int
    lib.ta_attention.argtypes = [LP, P, P, P, P, I64, I32, I32, I32, I32, P, P, P, P, P, P]
    lib.ta_attention_noalloc.restype = ctypes.c_int
    lib.ta_attention_noalloc.argtypes = [LP, P, P, P, P, I64, I32, I32, I32, I32, P, P, P, P]
    lib.ta_update_tail_klen.restype = ctypes.c_int
    lib.ta_update_tail_klen.argtypes = [P, P, I32, I32, I32, P, P]
    lib.ta_decode_append.restype = ctypes.c_int
    lib.ta_decode_append.argtypes = [P, P, P, P, I64, I64, P, I32, I32, I64, I32, I32, P, P, I32, P, I32, I32, P, P]
    lib.ta_plan_build.restype = ctypes.c_int
    lib.ta_plan_build.argtypes = [P, P, P, P, I32, I32, I32, I32, I32, I32, I64, P, I64,
                                  ctypes.POINTER(ctypes.c_int64), LP]
    lib.ta_schedule_tree.restype = ctypes.c_int
    lib.ta_schedule_tree.argtypes = [P, P, P, P, P, I32, I32, ctypes.POINTER(CostModelC), I32, I32, I32, P,
                                     ctypes.POINTER(ctypes.c_double)]
    version = lib.ta_abi_version()
    if version != ABI_VERSION:
        raise RuntimeError(f"kernel library ABI {version}, expected {ABI_VERSION}; rebuild it")
    _lib = lib
    return lib


def check(rc, what):
    if rc != 0:
        raise RuntimeError(f"{what} failed: {describe_status(rc)} (code {rc})")
