"""The C-ABI library: loads without a GPU and exports every symbol the header declares."""
import re
import subprocess
from pathlib import Path

import pytest

from tree_attention import _lib

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "tree_attn.h"


def declared_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\s*\*?\s*(ta_\w+)\s*\(", text, flags=re.M)))


def test_header_declarations_match_binding():
    assert declared_functions() == sorted(_lib.EXPORTS)


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in declared_functions():
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r" T (ta_\w+)$", out, flags=re.M))
    assert set(declared_functions()) <= exported


def test_abi_version_and_error_strings():
    lib = _lib.load()
    assert lib.ta_abi_version() == _lib.ABI_VERSION
    assert lib.ta_error_string(0) == b"ok"
    assert lib.ta_error_string(_lib.ERR_BOUNDS).startswith(b"plan index")


def test_argument_validation_without_gpu():
    """Rejected arguments return an error code before any CUDA call."""
    lib = _lib.load()
    layout = _lib.PlanLayout()
    layout.kstart_stride = 1
    assert lib.ta_segment(None, None, None, None, None, 0, 32, 8, 128, 1, None, None, None, None) == _lib.ERR_ARG
    # 6 query heads over 4 KV heads is not a GQA grouping
    assert lib.ta_segment(layout, 1024, None, None, None, 0, 6, 4, 128, 1, None, None, None,
                          None) == _lib.ERR_UNSUPPORTED
    assert lib.ta_merge(layout, 1024, None, None, None, None, 32, 8, 48, 1, None, None) == _lib.ERR_UNSUPPORTED
    assert lib.ta_update_tail_klen(None, None, -1, 0, 0, None, None) == _lib.ERR_ARG
    # an empty plan is a no-op
    assert lib.ta_segment(layout, 1024, None, None, None, 0, 32, 8, 128, 1, None, None, None, None) == 0
    # keys-in-lanes CTA counts: the per-class counts must add up to kn_ctas
    bad = _lib.PlanLayout.from_buffer_copy(layout)
    bad.kn_ctas = 3
    bad.kn_class_ctas[1] = 2
    assert lib.ta_segment(bad, 1024, None, None, None, 0, 32, 8, 128, 1, None, None, None, None) == _lib.ERR_ARG

    # the 16- to 64-row classes have no kernel in this build (checked after the pointers, which are
    # fake but aligned here: nothing is launched)
    reserved = _lib.PlanLayout.from_buffer_copy(layout)
    reserved.num_kn_tasks, reserved.num_kn_segs, reserved.kn_ctas = 1, 1, 1
    reserved.kn_class_ctas[2] = 1
    fake = 1 << 20
    assert lib.ta_segment(reserved, fake, fake, fake, fake, 0, 32, 8, 128, 1, fake, fake, None,
                          None) == _lib.ERR_UNSUPPORTED


def test_layout_struct_matches_header():
    import ctypes
    text = HEADER.read_text()
    body = text[text.index("typedef struct ta_plan_layout"):text.index("} ta_plan_layout;")]
    names = re.findall(r"int32_t (\w+)(?:\[(\d+)\])?;", body)
    fields = [(n, int(c) if c else 1) for n, c in names]
    assert [(f[0], getattr(f[1], "_length_", 1)) for f in _lib.PlanLayout._fields_] == fields
    assert ctypes.sizeof(_lib.PlanLayout) == 4 * sum(c for _, c in fields)


def test_decode_append_validation_without_gpu():
    """ta_decode_append rejects bad arguments before any CUDA call."""
    lib = _lib.load()
    bf16 = _lib.DTYPE_BF16

    def call(dtype=bf16, nreq=2, heads=8, dim=128, stride_r=1024, stride_h=128, ptr=4096, klen=None, tails=None,
             count=None, num_tails=0):
        return lib.ta_decode_append(ptr, ptr, ptr, ptr, stride_r, stride_h, ptr, nreq, heads, 64, dim, dtype, klen,
                                    tails, num_tails, count, 1, 4, None, None)

    assert call(dtype=7) == _lib.ERR_UNSUPPORTED
    assert call(dim=127) == _lib.ERR_ARG            # rows move as bf16 pairs
    assert call(stride_h=129) == _lib.ERR_ARG
    assert call(heads=0) == _lib.ERR_ARG
    assert call(ptr=4098) == _lib.ERR_ARG           # 2-byte aligned pointers
    assert call(klen=4096) == _lib.ERR_ARG          # a tail update without tail indices / count
    assert call(nreq=0) == 0                        # nothing to do, nothing launched


def test_noalloc_capacity_check_cannot_wrap_around():
    """ta_attention_noalloc bounds its size arithmetic before multiplying (no CUDA call is reached)."""
    lib = _lib.load()
    layout = _lib.PlanLayout()
    layout.kstart_stride = 1
    layout.num_partials = 2 ** 31 - 1
    # 2^31-1 partials x 2^30 query heads x 129 floats wraps a 64-bit size product: must still be rejected
    assert lib.ta_attention_noalloc(layout, None, None, None, None, 0, 2 ** 30, 1, 128, _lib.DTYPE_BF16, None,
                                    None, None, None) == _lib.ERR_TOO_LARGE
    # head sizes without a kernel are rejected before the size check
    assert lib.ta_attention_noalloc(layout, None, None, None, None, 0, 32, 8, 96, _lib.DTYPE_BF16, None,
                                    None, None, None) == _lib.ERR_UNSUPPORTED
