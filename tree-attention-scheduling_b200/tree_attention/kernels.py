"""Kernel entry points of the tree-attention decode path (B200, sm_100a).

Drop-in for the reference's ``src/tree_attention/kernels.py``:

* ``prepare(plan, q) -> PreparedPlan`` (kernels.py:86-141): physical jobs, the
  small-first stable sort, and the int32 arrays ``qids, kids, qlen, klen,
  slots, counts`` -- bit-identical to the reference -- in ONE device buffer
  uploaded with one host-to-device copy, plus this implementation's compact
  partial slots and kernel task lists in the same buffer.
* ``pack_kv(k, v)`` (kernels.py:144-145): ``[T, HK, D]`` K/V into the resident
  pool layout.  Both pools are token-major ``[HK, T, D]`` here (the reference
  keeps K as ``[HK, D, T]``); every key row is then one contiguous line, which
  is what the bulk-copy and TMA loads of the sm_100a kernels want.
* ``attention(q, k, v, prepared)`` / ``attention_matrix(q, kp, vp, prepared)``
  (kernels.py:148-168): the decode-step attention through the C ABI
  ``ta_attention`` (segment kernels + fused LSE merge) on the current CUDA
  stream.  Returns ``prepared.out``, a buffer owned by the plan and overwritten
  by the next call, exactly like the reference.
* ``CachedDecodePlan(prefix_plan, q, prefix_tokens, max_new_tokens)`` with
  ``update(generated)`` (kernels.py:171-186): the prompt plan plus one private
  tail job per request whose length is rewritten on the device each step.

There is no CPU or framework fallback: without the CUDA library every entry
point that launches work raises.
"""
from __future__ import annotations

import os
from dataclasses import dataclass, field
from math import ceil

import numpy as np
import torch

from . import _lib
from .schedule import Job, Plan, physical_jobs

# Query rows a small-group (SIMT) task covers; larger jobs go to the tensor-core
# kernel in tiles of TC_ROWS rows when it supports the shape.
SMALL_ROWS = 16
TC_ROWS = 256
# Reference sort key: jobs with more than 16 query rows run in the second phase
# (kernels.py:109-110).  Kept verbatim so the metadata is bit-identical.
_REF_SMALL_ROWS = 16

_DTYPES = {torch.bfloat16: _lib.DTYPE_BF16, torch.float16: _lib.DTYPE_F16}


def tc_supported(head_dim, dtype):
    """Whether the tcgen05 kernel handles this head size / dtype."""
    return head_dim == 128 and dtype in _DTYPES and os.environ.get("TREE_ATTN_DISABLE_TC") != "1" and _TC_BUILT


# Set once the tcgen05 kernel is part of the library.
_TC_BUILT = True


@dataclass
class PreparedPlan:
    """Device-resident plan: metadata, scratch and the reusable output (reference kernels.py:86-100)."""
    jobs: list
    small_jobs: int
    contiguous_k: bool
    contiguous_q: bool
    qids: torch.Tensor
    kids: torch.Tensor
    qlen: torch.Tensor
    klen: torch.Tensor
    slots: torch.Tensor
    counts: torch.Tensor
    part: torch.Tensor
    lse: torch.Tensor
    out: torch.Tensor
    # -- B200 additions ------------------------------------------------------
    metadata: torch.Tensor = None
    layout: _lib.PlanLayout = None
    slot_base: torch.Tensor = None
    cslots: torch.Tensor = None
    small_tasks: torch.Tensor = None
    tc_tasks: torch.Tensor = None
    status: torch.Tensor = None
    num_kv_heads: int = 0
    host_arrays: dict = field(default_factory=dict)


def _small_class(rows):
    return 0 if rows <= 4 else (1 if rows <= 8 else 2)


def build_metadata(jobs, num_requests, groups, use_tc):
    """Host-side metadata of a sorted physical job list (numpy int32 arrays).

    Returns the reference arrays (qids, kids, qlen, klen, slots, counts) and the
    B200 arrays (slot_base, cslots, small_tasks, tc_tasks, small_class_end).
    """
    njobs = len(jobs)
    maxr = max(len(j.requests) for j in jobs)
    contiguous_k = all(j.tokens[-1] - j.tokens[0] + 1 == len(j.tokens) for j in jobs)
    maxk = 1 if contiguous_k else max(len(j.tokens) for j in jobs)
    qids = np.zeros((njobs, maxr), dtype=np.int32)
    kids = np.zeros((njobs, maxk), dtype=np.int32)
    qlen = np.fromiter((len(j.requests) for j in jobs), dtype=np.int32, count=njobs)
    klen = np.fromiter((len(j.tokens) for j in jobs), dtype=np.int32, count=njobs)
    slot_base = np.zeros(njobs, dtype=np.int32)
    if njobs > 1:
        np.cumsum(qlen[:-1], out=slot_base[1:])
    per_request = [[] for _ in range(num_requests)]
    per_request_compact = [[] for _ in range(num_requests)]
    for i, job in enumerate(jobs):
        qids[i, :len(job.requests)] = job.requests
        if contiguous_k:
            kids[i, 0] = job.tokens[0]
        else:
            kids[i, :len(job.tokens)] = job.tokens
        base = int(slot_base[i])
        for j, r in enumerate(job.requests):
            per_request[r].append(i * maxr + j)
            per_request_compact[r].append(base + j)
    maxs = max(map(len, per_request))
    slots = np.zeros((num_requests, maxs), dtype=np.int32)
    cslots = np.zeros((num_requests, maxs), dtype=np.int32)
    for r in range(num_requests):
        slots[r, :len(per_request[r])] = per_request[r]
        cslots[r, :len(per_request_compact[r])] = per_request_compact[r]
    counts = np.fromiter((len(s) for s in per_request), dtype=np.int32, count=num_requests)

    small = [[], [], []]
    tc = []
    for i in range(njobs):
        rows = int(qlen[i]) * groups
        if rows <= SMALL_ROWS:
            small[_small_class(rows)].append((i, 0))
        elif use_tc:
            tc.extend((i, t) for t in range(ceil(rows / TC_ROWS)))
        else:
            for t in range(ceil(rows / SMALL_ROWS)):
                small[_small_class(min(SMALL_ROWS, rows - t * SMALL_ROWS))].append((i, t))
    class_end = np.cumsum([len(c) for c in small]).astype(np.int32)
    small_max_keys = max((int(klen[i]) for c in small for i, _ in c), default=0)
    small_tasks = np.array([t for c in small for t in c], dtype=np.int32).reshape(-1, 2)
    tc_tasks = np.array(tc, dtype=np.int32).reshape(-1, 2)
    return dict(qids=qids, kids=kids, qlen=qlen, klen=klen, slots=slots, counts=counts,
                slot_base=slot_base, cslots=cslots, small_tasks=small_tasks, tc_tasks=tc_tasks,
                small_class_end=class_end, small_max_keys=small_max_keys, contiguous_k=contiguous_k,
                num_partials=int(qlen.sum()))


_ORDER = ("qids", "kids", "qlen", "klen", "slots", "counts", "slot_base", "cslots", "small_tasks", "tc_tasks")


def prepare(plan, q, num_kv_heads=None):
    """Materialise ``plan`` for queries shaped like ``q`` ``[NREQ, HQ, D]`` (reference kernels.py:103-141).

    ``num_kv_heads`` defaults to ``plan.settings["kvheads"]``; a KV-head shard
    passes its local head count (the plan itself is head independent).
    """
    jobs = physical_jobs(plan.jobs)
    kvheads = num_kv_heads or plan.settings["kvheads"]
    nreq, hq, dim = q.shape
    if hq % kvheads:
        raise ValueError("Query heads must be divisible by KV heads")
    groups = hq // kvheads
    # Stable sort: small jobs (<= 16 query rows) first, as the reference does.
    jobs.sort(key=lambda job: len(job.requests) * groups > _REF_SMALL_ROWS)
    small_jobs = sum(len(job.requests) * groups <= _REF_SMALL_ROWS for job in jobs)
    for job in jobs:
        if not job.requests or not job.tokens:
            raise ValueError("Plan contains an empty job")
        if any(r < 0 or r >= nreq for r in job.requests):
            raise ValueError("Plan references a request outside the query batch")
    meta = build_metadata(jobs, nreq, groups, tc_supported(dim, q.dtype))
    if not meta["contiguous_k"]:
        raise ValueError("Physical jobs must read contiguous KV positions")

    offsets, pieces, offset = {}, [], 0
    for name in _ORDER:
        array = meta[name]
        offsets[name] = offset
        pieces.append(array.ravel())
        offset += array.size
    flat = np.concatenate(pieces) if offset else np.zeros(0, dtype=np.int32)
    device = q.device
    metadata = torch.from_numpy(flat).to(device)
    views = {name: metadata[offsets[name]:offsets[name] + meta[name].size].view(meta[name].shape)
             for name in _ORDER}

    layout = _lib.PlanLayout()
    layout.num_jobs = len(jobs)
    layout.max_requests = meta["qids"].shape[1]
    layout.max_slots = meta["slots"].shape[1]
    layout.num_requests = nreq
    layout.num_partials = meta["num_partials"]
    layout.num_small_tasks = meta["small_tasks"].shape[0]
    layout.num_tc_tasks = meta["tc_tasks"].shape[0]
    for i in range(3):
        layout.small_class_end[i] = int(meta["small_class_end"][i])
    layout.small_max_keys = meta["small_max_keys"]
    layout.kstart_stride = meta["kids"].shape[1]
    layout.off_qids = offsets["qids"]
    layout.off_kstart = offsets["kids"]
    layout.off_qlen = offsets["qlen"]
    layout.off_klen = offsets["klen"]
    layout.off_slots = offsets["slots"]
    layout.off_counts = offsets["counts"]
    layout.off_slot_base = offsets["slot_base"]
    layout.off_cslots = offsets["cslots"]
    layout.off_small_tasks = offsets["small_tasks"]
    layout.off_tc_tasks = offsets["tc_tasks"]

    rows = meta["num_partials"] * groups
    contiguous_q = all(j.requests[-1] - j.requests[0] + 1 == len(j.requests) for j in jobs)
    return PreparedPlan(
        jobs, small_jobs, True, contiguous_q,
        views["qids"], views["kids"], views["qlen"], views["klen"], views["slots"], views["counts"],
        torch.empty((kvheads, rows, dim), device=device, dtype=torch.float32),
        torch.empty((kvheads, rows), device=device, dtype=torch.float32),
        torch.empty_like(q),
        metadata=metadata, layout=layout, slot_base=views["slot_base"], cslots=views["cslots"],
        small_tasks=views["small_tasks"], tc_tasks=views["tc_tasks"],
        status=torch.zeros(1, device=device, dtype=torch.int32), num_kv_heads=kvheads,
        host_arrays=meta)


def pack_kv(k, v):
    """``[T, HK, D]`` K and V into the resident ``[HK, T, D]`` pools."""
    return k.permute(1, 0, 2).contiguous(), v.permute(1, 0, 2).contiguous()


def attention(q, k, v, prepared):
    """Attention of ``q`` over unpacked ``k, v`` ``[T, HK, D]`` (reference kernels.py:148-149)."""
    return attention_matrix(q, *pack_kv(k, v), prepared)


def _check_inputs(q, kp, vp, p):
    if q.dim() != 3 or kp.dim() != 3 or vp.dim() != 3:
        raise ValueError("q must be [NREQ, HQ, D] and the pools [HK, T, D]")
    if q.dtype not in _DTYPES or kp.dtype != q.dtype or vp.dtype != q.dtype:
        raise ValueError("q, K and V must share one dtype, bfloat16 or float16")
    if not (q.is_cuda and kp.is_cuda and vp.is_cuda):
        raise ValueError("tree attention runs on CUDA tensors only")
    nreq, hq, dim = q.shape
    hk, tokens, kdim = kp.shape
    if kdim != dim or tuple(vp.shape) != tuple(kp.shape):
        raise ValueError(f"pools must be [HK, T, D] with D={dim}; got K {tuple(kp.shape)}, V {tuple(vp.shape)}")
    if hq % hk or hk != p.num_kv_heads:
        raise ValueError(f"plan was prepared for {p.num_kv_heads} KV heads, pools have {hk}")
    if nreq != p.layout.num_requests or tuple(p.out.shape) != tuple(q.shape) or p.out.dtype != q.dtype:
        raise ValueError("queries do not match the prepared plan")
    if not (kp.is_contiguous() and vp.is_contiguous()):
        raise ValueError("K/V pools must be contiguous [HK, T, D]")


def attention_matrix(q, kp, vp, prepared, out_lse=None):
    """Decode-step attention on resident pools ``kp, vp`` ``[HK, T, D]`` (reference kernels.py:152-168).

    Returns ``prepared.out`` (owned by the plan, overwritten by the next call).
    ``out_lse`` (``[NREQ, HQ]`` float32, optional) receives the merged LSE.
    """
    p = prepared
    _check_inputs(q, kp, vp, p)
    if not q.is_contiguous():
        q = q.contiguous()
    lib = _lib.load()
    stream = torch.cuda.current_stream(q.device).cuda_stream
    rc = lib.ta_attention(
        p.layout, p.metadata.data_ptr(), q.data_ptr(), kp.data_ptr(), vp.data_ptr(), kp.shape[1],
        q.shape[1], kp.shape[0], q.shape[2], _DTYPES[q.dtype], p.part.data_ptr(), p.lse.data_ptr(),
        p.out.data_ptr(), out_lse.data_ptr() if out_lse is not None else None, p.status.data_ptr(), stream)
    _lib.check(rc, "ta_attention")
    if os.environ.get("TREE_ATTN_CHECK") == "1":
        check_status(p)
    return p.out


def check_status(prepared):
    """Synchronise and raise if a kernel recorded a device-side error for this plan."""
    code = int(prepared.status.item())
    if code:
        prepared.status.zero_()
        raise RuntimeError(f"tree-attention device status: {_lib.describe_status(code)} (code {code})")


class CachedDecodePlan:
    """A prompt schedule plus one contiguous growing KV tail per request (reference kernels.py:171-186)."""

    def __init__(self, prefix_plan, q, prefix_tokens, max_new_tokens, num_kv_heads=None):
        tails = [Job((r,), tuple(range(prefix_tokens + r * max_new_tokens,
                                       prefix_tokens + (r + 1) * max_new_tokens)))
                 for r in range(q.shape[0])]
        plan = Plan(prefix_plan.jobs + tails, prefix_plan.method, prefix_plan.estimated_us, prefix_plan.settings)
        self.prepared = prepare(plan, q, num_kv_heads)
        ordered = self.prepared.jobs
        tail_ids = [i for i, job in enumerate(ordered) if job.tokens[0] >= prefix_tokens]
        self.tail_indices = torch.tensor(tail_ids, device=q.device, dtype=torch.int32)

    def update(self, generated_tokens):
        """Set every tail's length to ``generated_tokens`` on the device; returns the plan."""
        p = self.prepared
        lib = _lib.load()
        stream = torch.cuda.current_stream(p.klen.device).cuda_stream
        rc = lib.ta_update_tail_klen(p.klen.data_ptr(), self.tail_indices.data_ptr(), self.tail_indices.numel(),
                                     int(generated_tokens), p.layout.num_jobs, p.status.data_ptr(), stream)
        _lib.check(rc, "ta_update_tail_klen")
        return p
