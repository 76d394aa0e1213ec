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

import ctypes
import os
from dataclasses import dataclass, field
from itertools import chain
from math import ceil

import numpy as np
import torch

from . import _lib
from .schedule import Job, Plan, physical_jobs

# Routing of a job's query rows (requests x GQA group) for head_dim 128:
# up to KN_ROWS rows run on the persistent keys-in-lanes tcgen05 kernel
# (queries are the MMA N dimension), more rows on the query-tile tcgen05 kernel
# in pairs of 128-row tiles (TC_ROWS).  Other head sizes use the SIMT kernel in
# tiles of SMALL_ROWS rows.  The 16-row threshold (the reference's own split,
# kernels.py:109-110) measured best on the evaluation grid: at 32 or 64 the
# keys-in-lanes kernel re-reads a shared segment once per 8-row segment.
KN_ROWS = 16
TC_ROWS = 256
SMALL_ROWS = 16
KEY_TILE = 128
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
    pieces: torch.Tensor = None
    cslots: torch.Tensor = None
    small_tasks: torch.Tensor = None
    tc_tasks: torch.Tensor = None
    kn_tasks: torch.Tensor = None
    status: torch.Tensor = None
    num_kv_heads: int = 0
    host_arrays: dict = field(default_factory=dict)


def _small_class(rows):
    return 0 if rows <= 4 else (1 if rows <= 8 else 2)


def _route(rows, use_tc):
    if not use_tc:
        return "simt"
    return "kn" if rows <= KN_ROWS else "tc"


def _tiles(keys):
    return max(1, -(-keys // KEY_TILE))


def split_pieces(jobs, groups, heads, use_tc, sms, no_split_from=None, tc_max_ctas=None, levels=None):
    """Cut jobs into execution pieces ``(job, key_offset, keys)`` so the kernels fill the GPU.

    A piece is a contiguous key range of one job with its own partial slots;
    the merge combines a request's partials across pieces exactly as across
    jobs, so splitting changes the work distribution, never the result beyond
    float rounding.  Keys-in-lanes jobs are cut so no piece holds more than
    about half a CTA's share of all key tiles; query-tile jobs are cut while
    their CTAs still fit one wave on ``sms`` SMs, a whole level of the longest
    pieces at a time.  Jobs whose first position is
    at or past ``no_split_from`` (the growing decode tails) stay whole.
    ``tc_max_ctas`` caps the query-tile CTAs below ``sms``; ``levels``, if a
    list, receives ``(query-tile CTAs, longest piece in key tiles)`` of every
    level the cutting passes through.
    """
    n = len(jobs)
    rows = [len(j.requests) * groups for j in jobs]
    route = [_route(r, use_tc) for r in rows]
    keys = [len(j.tokens) for j in jobs]
    splittable = [no_split_from is None or j.tokens[0] < no_split_from for j in jobs]
    count = [1] * n

    kn = [i for i in range(n) if route[i] == "kn"]
    if kn:
        total = sum(_tiles(keys[i]) for i in kn) * heads
        cap = max(2, -(-total // (2 * sms)))
        for i in kn:
            if splittable[i] and _tiles(keys[i]) > cap:
                count[i] = -(-_tiles(keys[i]) // cap)

    tc = [i for i in range(n) if route[i] == "tc"]
    if tc:
        # Cut level by level: every job whose pieces are the longest takes one
        # more piece, as long as all of them can and the query-tile CTAs still
        # fit one wave.  A partial level would add CTAs without shortening the
        # longest piece; the SMs it leaves free run the small-group kernel
        # beside the query-tile kernel.
        pairs = {i: -(-rows[i] // TC_ROWS) * heads for i in tc}
        ctas = sum(pairs.values())
        limit = sms if tc_max_ctas is None else min(sms, tc_max_ctas)
        while True:
            longest = max(-(-_tiles(keys[i]) // count[i]) for i in tc)
            if levels is not None:
                levels.append((ctas, longest))
            level = [i for i in tc if -(-_tiles(keys[i]) // count[i]) == longest]
            if not all(splittable[i] and _tiles(keys[i]) / (count[i] + 1) >= 2 for i in level):
                break
            extra = sum(pairs[i] for i in level)
            if ctas + extra > limit:
                break
            for i in level:
                count[i] += 1
            ctas += extra

    pieces = []
    for i in range(n):
        tiles = _tiles(keys[i])
        per = -(-tiles // count[i]) * KEY_TILE
        offset = 0
        while True:
            take = min(per, keys[i] - offset)
            pieces.append((i, offset, take))
            offset += take
            if offset >= keys[i]:
                break
    return pieces, route, rows


# Keys-in-lanes tasks of at most KN_DUAL_ROWS query rows run KN_DUAL_CTAS
# persistent CTAs per SM (each with a single K and V stage), so two CTAs'
# softmax chains interleave on every SM.
KN_DUAL_ROWS = 8
KN_DUAL_CTAS = 2
# Query rows of one keys-in-lanes segment: larger jobs are cut into segments
# of whole requests (each re-reads the job's K/V tiles, mostly from L2).
KN_TASK_ROWS = 8
# Row classes of the keys-in-lanes launches (the kernel's N dimension is
# max(16, class rows)).
KN_CLASS_ROWS = (4, 8, 16, 32, 64)


def kn_class(rows):
    """Row class of a keys-in-lanes task with `rows` query rows."""
    return next(c for c, r in enumerate(KN_CLASS_ROWS) if rows <= r)
KN_BOX = 32          # keys-in-lanes TMA box height: packed segments start on 32-key boundaries
KN_PACK_ROWS = 8    # query rows of a packed tile
KN_PACK_SEGS = 4     # segments of a packed tile


def pack_segments(items):
    """Group keys-in-lanes segments into tasks.

    ``items`` are ``(head, rows, first_partial_row, k0, keys, job_flags, first_request,
    request_offset)``.  A segment of more
    than one 128-key tile is a task of its own; shorter ones are packed, best
    fit by their 32-key-rounded span, into tiles of 128 keys, at most
    KN_PACK_SEGS segments and KN_PACK_ROWS query rows each (a segment of more
    rows stays alone).  Returns a list of tasks, each a list of items.
    """
    tasks, open_bins = [], {32: [], 64: [], 96: []}    # remaining span -> bins
    packable = []
    for item in items:
        span = -(-item[4] // KN_BOX) * KN_BOX
        if item[4] > KEY_TILE or span >= KEY_TILE or item[1] > KN_PACK_ROWS // 2:
            tasks.append([item])
        else:
            packable.append((span, item))
    packable.sort(key=lambda x: -x[0])
    for span, item in packable:
        placed = False
        for free in (32, 64, 96):
            if free < span:
                continue
            for b, (segs, used_rows) in enumerate(open_bins[free]):
                if used_rows + item[1] <= KN_PACK_ROWS and len(segs) < KN_PACK_SEGS:
                    open_bins[free].pop(b)
                    segs.append(item)
                    left = free - span
                    if left and len(segs) < KN_PACK_SEGS:
                        open_bins[left].append((segs, used_rows + item[1]))
                    else:
                        tasks.append(segs)
                    placed = True
                    break
                break                     # rows are uniform enough: only the first bin is tried
            if placed:
                break
        if not placed:
            left = KEY_TILE - span
            if left:
                open_bins[left].append(([item], item[1]))
            else:
                tasks.append([item])
    for free in (32, 64, 96):
        tasks.extend(segs for segs, _ in open_bins[free])
    return tasks


# Step-time model that picks how far query-tile jobs are cut (tenths of a
# microsecond, from steady-state timelines of the two kernels on one B200):
# a query-tile CTA costs TC_FIXED plus TC_PER_TILE per K/V tile of its piece;
# a keys-in-lanes CTA costs KN_FIXED plus KN_PER_TASK per task it runs.
TC_FIXED, TC_PER_TILE, KN_FIXED, KN_PER_TASK = 70, 22, 25, 35


def kn_class_counts(jobs, piece_list, route, rows, groups, heads):
    """Keys-in-lanes tasks per row class of a piece list (the packing of ``build_metadata``)."""
    chunk = max(groups, KN_TASK_ROWS // groups * groups)
    items = []
    for i, offset, take in piece_list:
        if route[i] == "kn":
            for h in range(heads):
                for r0 in range(0, rows[i], chunk):
                    items.append((h, min(chunk, rows[i] - r0), 0, 0, take, 0, -1, 0))
    counts = [0] * len(KN_CLASS_ROWS)
    for task in pack_segments(items):
        counts[kn_class(sum(item[1] for item in task))] += 1
    return counts


def choose_tc_level(levels, class_counts, sms):
    """Cut level of the query-tile jobs and keys-in-lanes placement with the lowest modelled step time.

    ``levels``: ``(query-tile CTAs, longest piece in tiles)`` per cut level
    (``split_pieces``), coarsest first.  Two placements of the keys-in-lanes
    tasks are weighed: after the query tiles, each class over
    ``min(KN_DUAL_CTAS * sms, tasks)`` CTAs (the default), or - with one row
    class - beside them, on ``KN_DUAL_CTAS`` CTAs per SM the query tiles leave
    free, all placed when the launch is (CTAs placed later wait for the
    query-tile grid to finish).  Returns ``(cap, beside)``: the query-tile CTA
    cap for ``split_pieces`` (None: no cap) and, for the beside placement, the
    query-tile CTA count the keys-in-lanes CTAs are sized against (else None).
    Ties keep more query-tile CTAs, then the default placement.
    """
    if not levels:
        return None, None
    used = [c for c in range(len(KN_CLASS_ROWS)) if class_counts[c]]
    dual = {c: KN_DUAL_CTAS if KN_CLASS_ROWS[c] <= KN_DUAL_ROWS else 1 for c in used}
    best = None
    for index, (ctas, longest) in enumerate(levels):
        t_tc = TC_FIXED + TC_PER_TILE * longest
        options = []
        if not used:
            options.append((t_tc, 0))
        else:
            rounds = max(-(-class_counts[c] // min(dual[c] * sms, class_counts[c])) for c in used)
            options.append((t_tc + KN_FIXED + KN_PER_TASK * rounds, 0))
            if len(used) == 1 and sms > ctas:
                c = used[0]
                side = min(dual[c] * (sms - ctas), class_counts[c])
                options.append((max(t_tc, KN_FIXED + KN_PER_TASK * -(-class_counts[c] // side)), 1))
        for t, mode in options:
            key = (t, -index, mode)
            if best is None or key < best[0]:
                best = (key, index, mode)
    _, index, mode = best
    cap = None if index == len(levels) - 1 else levels[index][0]
    return cap, (levels[index][0] if mode else None)


def assign_lpt(costs, bins):
    """Longest-processing-time assignment of tasks to ``bins`` persistent CTAs.

    Returns (offsets [bins + 1], order): CTA b runs ``order[offsets[b]:offsets[b + 1]]``.
    """
    import heapq
    heap = [(0, b) for b in range(bins)]
    lists = [[] for _ in range(bins)]
    for task in sorted(range(len(costs)), key=lambda t: -costs[t]):
        load, b = heapq.heappop(heap)
        lists[b].append(task)
        heapq.heappush(heap, (load + costs[task], b))
    offsets = np.zeros(bins + 1, dtype=np.int32)
    np.cumsum([len(x) for x in lists], out=offsets[1:])
    order = np.array([t for x in lists for t in x], dtype=np.int32)
    return offsets, order


def build_metadata(jobs, num_requests, groups, use_tc, heads=1, sms=148, no_split_from=None):
    """Host-side metadata of a sorted physical job list (numpy int32 arrays).

    Returns the reference arrays (qids, kids, qlen, klen, slots, counts) and the
    B200 arrays: execution pieces [P, 4] (job, key offset, keys, first partial
    slot), per-request partial counts and slots over pieces, SIMT tasks (piece,
    16-row tile) in three row classes, query-tile tasks (piece, 256-row pair)
    and the keys-in-lanes tasks (headers in persistent-CTA order, segment records).

    This is the readable statement of the construction; ``prepare`` runs the
    library's native ``ta_plan_build`` (``csrc/plan.cpp``), which tests hold
    bit-identical to it (``flatten_metadata`` of this result).
    """
    njobs = len(jobs)
    maxr = max(len(j.requests) for j in jobs)
    contiguous_k = all(j.tokens[-1] - j.tokens[0] + 1 == len(j.tokens) for j in jobs)
    maxk = 1 if contiguous_k else max(len(j.tokens) for j in jobs)
    qids = np.zeros((njobs, maxr), dtype=np.int32)
    kids = np.zeros((njobs, maxk), dtype=np.int32)
    qlen = np.fromiter((len(j.requests) for j in jobs), dtype=np.int32, count=njobs)
    klen = np.fromiter((len(j.tokens) for j in jobs), dtype=np.int32, count=njobs)
    per_request = [[] for _ in range(num_requests)]
    for i, job in enumerate(jobs):
        qids[i, :len(job.requests)] = job.requests
        if contiguous_k:
            kids[i, 0] = job.tokens[0]
        else:
            kids[i, :len(job.tokens)] = job.tokens
        for j, r in enumerate(job.requests):
            per_request[r].append(i * maxr + j)
    maxs = max(map(len, per_request))
    slots = np.zeros((num_requests, maxs), dtype=np.int32)
    for r in range(num_requests):
        slots[r, :len(per_request[r])] = per_request[r]
    counts = np.fromiter((len(s) for s in per_request), dtype=np.int32, count=num_requests)

    levels = []
    piece_list, route, rows = split_pieces(jobs, groups, heads, use_tc, sms, no_split_from, levels=levels)
    tc_cap, kn_beside = choose_tc_level(levels, kn_class_counts(jobs, piece_list, route, rows, groups, heads), sms)
    if tc_cap is not None:
        piece_list, route, rows = split_pieces(jobs, groups, heads, use_tc, sms, no_split_from, tc_max_ctas=tc_cap)
    npieces = len(piece_list)
    pieces = np.zeros((npieces, 4), dtype=np.int32)
    per_request_p = [[] for _ in range(num_requests)]
    slot = 0
    for p, (i, offset, take) in enumerate(piece_list):
        pieces[p] = (i, offset, take, slot)
        for j, r in enumerate(jobs[i].requests):
            per_request_p[r].append(slot + j)
        slot += len(jobs[i].requests)
    maxp = max(map(len, per_request_p))
    cslots = np.zeros((num_requests, maxp), dtype=np.int32)
    for r in range(num_requests):
        cslots[r, :len(per_request_p[r])] = per_request_p[r]
    pcounts = np.fromiter((len(s) for s in per_request_p), dtype=np.int32, count=num_requests)

    small = [[], [], []]
    tc = []
    items = []          # keys-in-lanes segments: one per (piece, KV head)
    for p, (i, offset, take) in enumerate(piece_list):
        if route[i] == "kn":
            growing = int(no_split_from is not None and jobs[i].tokens[0] >= no_split_from)
            reqs = jobs[i].requests
            q0 = reqs[0] if reqs[-1] - reqs[0] + 1 == len(reqs) else -1
            for h in range(heads):
                # at most KN_TASK_ROWS rows per segment (whole requests): one
                # launch class for nearly every plan, and short softmax chains
                chunk = max(groups, KN_TASK_ROWS // groups * groups)
                for r0 in range(0, rows[i], chunk):
                    c0 = r0 // groups
                    items.append((h, min(chunk, rows[i] - r0), int(pieces[p, 3]) * groups + r0,
                                  jobs[i].tokens[0] + offset, take, i | (growing << 30),
                                  q0 + c0 if q0 >= 0 else -1, c0))
        elif route[i] == "tc":
            reqs = jobs[i].requests
            q0 = reqs[0] if reqs[-1] - reqs[0] + 1 == len(reqs) else -1
            tc.extend((p, t, q0, 0) for t in range(ceil(rows[i] / TC_ROWS)))
        else:
            for t in range(ceil(rows[i] / SMALL_ROWS)):
                small[_small_class(min(SMALL_ROWS, rows[i] - t * SMALL_ROWS))].append((p, t))
    class_end = np.cumsum([len(c) for c in small]).astype(np.int32)
    small_max_keys = max((piece_list[p][2] for c in small for p, _ in c), default=0)
    small_tasks = np.array([t for c in small for t in c], dtype=np.int32).reshape(-1, 2)
    tc_tasks = np.array(tc, dtype=np.int32).reshape(-1, 4)
    tasks = pack_segments(items)
    segs = []
    by_class = [[] for _ in KN_CLASS_ROWS]          # (header, cost) per row class
    for task in tasks:
        header = (len(segs), len(task), 0, 0)
        row0, kt = 0, 0
        for h, r, first_row, k0, keys, job, q0, qofs in task:
            segs.append((h, row0, r, first_row, k0, kt if len(task) > 1 else 0, keys, job, q0, qofs, 0, 0))
            row0 += r
            kt += -(-keys // KN_BOX) * KN_BOX
        by_class[kn_class(row0)].append((header, _tiles(max(s[4] for s in task)) + 1))
    # one launch per non-empty class, each balanced over its own CTAs
    kn_class_ctas = np.zeros(len(KN_CLASS_ROWS), dtype=np.int32)
    offsets, ordered = [0], []
    for c, entries in enumerate(by_class):
        if not entries:
            continue
        per_sm = KN_DUAL_CTAS if KN_CLASS_ROWS[c] <= KN_DUAL_ROWS else 1
        # beside the query tiles: on the SMs they leave free
        ctas = min(per_sm * (sms if kn_beside is None else sms - kn_beside), len(entries))
        offs, order = assign_lpt([cost for _, cost in entries], ctas)
        base = len(ordered)
        offsets.extend(int(o) + base for o in offs[1:])
        ordered.extend(entries[i][0] for i in order)
        kn_class_ctas[c] = ctas
    kn_ctas = int(kn_class_ctas.sum())
    kn_offsets = np.array(offsets, dtype=np.int32)
    kn_tasks = np.array(ordered, dtype=np.int32).reshape(-1, 4)
    kn_segs = np.array(segs, dtype=np.int32).reshape(-1, 12)
    return dict(qids=qids, kids=kids, qlen=qlen, klen=klen, slots=slots, counts=counts,
                pieces=pieces, pcounts=pcounts, cslots=cslots, small_tasks=small_tasks, tc_tasks=tc_tasks,
                kn_offsets=kn_offsets, kn_tasks=kn_tasks, kn_segs=kn_segs, small_class_end=class_end,
                small_max_keys=small_max_keys, kn_ctas=kn_ctas, kn_class_ctas=kn_class_ctas, contiguous_k=contiguous_k,
                num_partials=slot)


_ORDER = ("qids", "kids", "qlen", "klen", "slots", "counts", "pieces", "pcounts", "cslots", "small_tasks",
          "tc_tasks", "kn_offsets", "kn_tasks", "kn_segs")


def _sm_count(device):
    if device.type == "cuda" and torch.cuda.is_available():
        return torch.cuda.get_device_properties(device).multi_processor_count
    return 148


_SHAPES = {
    "qids": lambda L: (L.num_jobs, L.max_requests), "kids": lambda L: (L.num_jobs, L.kstart_stride),
    "qlen": lambda L: (L.num_jobs,), "klen": lambda L: (L.num_jobs,),
    "slots": lambda L: (L.num_requests, L.max_slots), "counts": lambda L: (L.num_requests,),
    "pieces": lambda L: (L.num_pieces, 4), "pcounts": lambda L: (L.num_requests,),
    "cslots": lambda L: (L.num_requests, L.max_pslots), "small_tasks": lambda L: (L.num_small_tasks, 2),
    "tc_tasks": lambda L: (L.num_tc_tasks, 4), "kn_offsets": lambda L: (L.kn_ctas + 1,),
    "kn_tasks": lambda L: (L.num_kn_tasks, 4), "kn_segs": lambda L: (L.num_kn_segs, 12)}
_OFFSET_FIELD = {name: "off_" + ("kstart" if name == "kids" else name) for name in _ORDER}


def flatten_metadata(meta, num_requests):
    """``build_metadata``'s arrays as ``prepare``'s single int32 buffer and its layout.

    Every array starts on a 16-byte boundary, in ``_ORDER``.  The native builder
    produces exactly this buffer; tests compare the two.
    """
    offsets, parts, offset = {}, [], 0
    for name in _ORDER:
        array = meta[name]
        pad = -offset % 4                 # every array starts on a 16-byte boundary
        if pad:
            parts.append(np.zeros(pad, dtype=np.int32))
            offset += pad
        offsets[name] = offset
        parts.append(array.ravel())
        offset += array.size
    flat = np.concatenate(parts) if offset else np.zeros(0, dtype=np.int32)
    layout = _lib.PlanLayout()
    layout.num_jobs = meta["qids"].shape[0]
    layout.max_requests = meta["qids"].shape[1]
    layout.max_slots = meta["slots"].shape[1]
    layout.num_requests = num_requests
    layout.num_pieces = meta["pieces"].shape[0]
    layout.num_partials = meta["num_partials"]
    layout.max_pslots = meta["cslots"].shape[1]
    layout.num_small_tasks = meta["small_tasks"].shape[0]
    layout.num_tc_tasks = meta["tc_tasks"].shape[0]
    layout.num_kn_tasks = meta["kn_tasks"].shape[0]
    layout.num_kn_segs = meta["kn_segs"].shape[0]
    layout.kn_ctas = meta["kn_ctas"]
    for c in range(len(KN_CLASS_ROWS)):
        layout.kn_class_ctas[c] = int(meta["kn_class_ctas"][c])
    for i in range(3):
        layout.small_class_end[i] = int(meta["small_class_end"][i])
    layout.small_max_keys = meta["small_max_keys"]
    layout.kstart_stride = meta["kids"].shape[1]
    for name in _ORDER:
        setattr(layout, _OFFSET_FIELD[name], offsets[name])
    return flat, layout


def _native_metadata(jobs, num_requests, groups, use_tc, heads, sms, no_split_from):
    """``build_metadata`` + ``flatten_metadata`` by the library's ``ta_plan_build``.

    Returns (flat int32 buffer, layout, the arrays as numpy views of the buffer).
    """
    lib = _lib.load()
    njobs = len(jobs)
    nq = np.fromiter((len(j.requests) for j in jobs), dtype=np.int32, count=njobs)
    req_offsets = np.zeros(njobs + 1, dtype=np.int32)
    np.cumsum(nq, out=req_offsets[1:])
    reqs = np.fromiter(chain.from_iterable(j.requests for j in jobs), dtype=np.int32, count=int(req_offsets[-1]))
    k0 = np.fromiter((j.tokens[0] for j in jobs), dtype=np.int32, count=njobs)
    keys = np.fromiter((len(j.tokens) for j in jobs), dtype=np.int32, count=njobs)
    layout = _lib.PlanLayout()
    size = ctypes.c_int64(0)
    capacity = 8 * (njobs + len(reqs)) * max(1, heads) + 4 * num_requests * 8 + 1024
    for _ in range(2):
        flat = np.empty(capacity, dtype=np.int32)
        rc = lib.ta_plan_build(req_offsets.ctypes.data, reqs.ctypes.data, k0.ctypes.data, keys.ctypes.data, njobs,
                               num_requests, groups, int(use_tc), heads, sms,
                               -1 if no_split_from is None else int(no_split_from), flat.ctypes.data, capacity,
                               ctypes.byref(size), ctypes.byref(layout))
        if rc != _lib.ERR_TOO_LARGE:
            break
        capacity = size.value
    _lib.check(rc, "ta_plan_build")
    flat = flat[:size.value]
    meta = {name: flat[getattr(layout, _OFFSET_FIELD[name]):].ravel()[:int(np.prod(_SHAPES[name](layout)))]
            .reshape(_SHAPES[name](layout)) for name in _ORDER}
    meta.update(small_class_end=np.array(layout.small_class_end[:], dtype=np.int32),
                small_max_keys=layout.small_max_keys, kn_ctas=layout.kn_ctas,
                kn_class_ctas=np.array(layout.kn_class_ctas[:], dtype=np.int32), contiguous_k=True,
                num_partials=layout.num_partials)
    return flat, layout, meta


def prepare(plan, q, num_kv_heads=None, _no_split_from=None):
    """Materialise ``plan`` for queries shaped like ``q`` ``[NREQ, HQ, D]`` (reference kernels.py:103-141).

    ``num_kv_heads`` defaults to ``plan.settings["kvheads"]``; a KV-head shard
    passes its local head count (the plan itself is head independent).  The
    arrays are built by the library's native ``ta_plan_build`` (the construction
    ``build_metadata`` states) and uploaded with one host-to-device copy.
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
    if not jobs:
        raise ValueError("Plan contains no jobs")
    if not all(job.requests and job.tokens for job in jobs):
        raise ValueError("Plan contains an empty job")
    if not all(job.tokens[-1] - job.tokens[0] + 1 == len(job.tokens) for job in jobs):
        raise ValueError("Physical jobs must read contiguous KV positions")
    lo = min(min(job.requests) for job in jobs)
    hi = max(max(job.requests) for job in jobs)
    if lo < 0 or hi >= nreq:
        raise ValueError("Plan references a request outside the query batch")
    flat, layout, meta = _native_metadata(jobs, nreq, groups, tc_supported(dim, q.dtype), kvheads,
                                          _sm_count(q.device), _no_split_from)
    device = q.device
    metadata = torch.from_numpy(flat).to(device)
    views = {name: metadata[getattr(layout, _OFFSET_FIELD[name]):][:meta[name].size].view(meta[name].shape)
             for name in _ORDER}

    rows = meta["num_partials"] * groups
    contiguous_q = all(j.requests[-1] - j.requests[0] + 1 == len(j.requests) for j in jobs)
    return PreparedPlan(
        jobs, small_jobs, True, contiguous_q,
        views["qids"], views["kids"], views["qlen"], views["klen"], views["slots"], views["counts"],
        torch.empty((kvheads, rows, dim), device=device, dtype=torch.float32),
        torch.empty((kvheads, rows), device=device, dtype=torch.float32),
        torch.empty_like(q),
        metadata=metadata, layout=layout, pieces=views["pieces"], cslots=views["cslots"],
        small_tasks=views["small_tasks"], tc_tasks=views["tc_tasks"], kn_tasks=views["kn_tasks"],
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


def append_kv(kp, vp, k_new, v_new, targets, status=None, tails=None):
    """Write one decode step's new K/V rows into the resident pools, in one launch (``ta_decode_append``).

    ``k_new``/``v_new`` are ``[NREQ, HK, D]`` (rows contiguous, any request/head
    strides), ``targets`` the int64 pool positions ``[NREQ]`` on the device: the
    reference's ``kp.index_copy_`` / ``vp.index_copy_`` (qwen.py:89-90).
    ``tails = (cached_plan, count, offset)`` also sets every tail length of a
    ``CachedDecodePlan`` to ``count + offset`` (``count`` a device int64 tensor
    of one element) in the same launch.  Out-of-range targets are skipped and
    recorded in ``status`` (default: the cached plan's).
    """
    hk, tokens, dim = kp.shape
    nreq = k_new.shape[0]
    if (vp.shape != kp.shape or k_new.shape != (nreq, hk, dim) or v_new.shape != k_new.shape
            or k_new.stride() != v_new.stride() or k_new.stride(2) != 1
            or not (kp.is_contiguous() and vp.is_contiguous())):
        raise ValueError("append_kv wants contiguous [HK, T, D] pools and [NREQ, HK, D] rows")
    if not (k_new.dtype == v_new.dtype == kp.dtype == vp.dtype) or kp.dtype not in _DTYPES:
        raise ValueError("append_kv: pools and rows must share one dtype, bfloat16 or float16")
    if targets.dtype != torch.int64 or targets.shape != (nreq,):
        raise ValueError("append_kv: targets must be int64 [NREQ]")
    # every pointer the kernel dereferences must be memory of the pools' GPU
    device = kp.device
    if device.type != "cuda" or any(t.device != device for t in (vp, k_new, v_new, targets)):
        raise ValueError("append_kv: pools, rows and targets must be CUDA tensors on one device")
    if status is not None and (status.device != device or status.dtype != torch.int32 or status.numel() < 1):
        raise ValueError("append_kv: status must be an int32 CUDA tensor on the pools' device")
    lib = _lib.load()
    klen = tail_ids = count = None
    offset = num_tails = num_jobs = 0
    if tails is not None:
        cached, count_t, offset = tails
        if count_t.device != device or count_t.dtype != torch.int64 or count_t.numel() < 1:
            raise ValueError("append_kv: the step count must be an int64 tensor of at least one element "
                             "on the pools' device")
        if cached.tail_indices.device != device or cached.tail_indices.dtype != torch.int32:
            raise ValueError("append_kv: the cached plan's tail indices must be int32 on the pools' device")
        p = cached.prepared
        if p.klen.device != device:
            raise ValueError("append_kv: the cached plan lives on another device than the pools")
        klen, tail_ids, count = p.klen.data_ptr(), cached.tail_indices.data_ptr(), count_t.data_ptr()
        num_tails, num_jobs = cached.tail_indices.numel(), p.layout.num_jobs
        status = p.status if status is None else status
    stream = torch.cuda.current_stream(kp.device).cuda_stream
    rc = lib.ta_decode_append(kp.data_ptr(), vp.data_ptr(), k_new.data_ptr(), v_new.data_ptr(), k_new.stride(0),
                              k_new.stride(1), targets.data_ptr(), nreq, hk, tokens, dim, _DTYPES[kp.dtype], klen,
                              tail_ids, num_tails, count, int(offset), num_jobs,
                              None if status is None else status.data_ptr(), stream)
    _lib.check(rc, "ta_decode_append")


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
        self.prepared = prepare(plan, q, num_kv_heads, _no_split_from=prefix_tokens)
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
