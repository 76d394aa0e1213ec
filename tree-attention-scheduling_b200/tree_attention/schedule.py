"""Grouping of (request set x KV segment) jobs over a radix tree.

Public API and plans follow the reference's ``src/tree_attention/schedule.py``:

* ``Job`` / ``physical_jobs`` (schedule.py:7-26): a job is a set of requests
  attending over a run of physical positions; ``physical_jobs`` cuts a job at
  every discontinuity so each piece is one contiguous KV read.
* ``CostModel`` (schedule.py:29-52): analytical roofline price of one physical
  job: ``max(flops / cube_flops, reads / bandwidth) + task_us * qtiles * kvheads
  + partial / bandwidth + merge_us * |R|`` with query-row and key-tile padding.
* ``Plan`` (schedule.py:55-69): jobs, method, estimated cost, settings;
  ``validate`` checks that the jobs partition every request's context exactly.
* ``schedule`` (schedule.py:72-151): ``request`` (one job per request),
  ``fixed`` (one job per node), ``greedy`` (per child, push the child's requests
  down with the parent's tokens when that is cheaper) and ``cube`` (exact subset
  DP over how many descendant requests are detached at every node), then tiling
  by ``max_query_rows // G`` requests x ``kv_split`` tokens.

For an identical ``CostModel`` the job list (order and content) and
``estimated_us`` are bit-identical to the reference: costs are summed in the
same order with ``sum()``, ties are broken the same way.  Unlike the reference,
the planner keeps token sequences as run-length tuples ``((start, length), ...)``
so the dynamic program hashes a few runs instead of thousands of positions.

``CostModel.b200()`` returns constants re-fitted to the B200 kernels of this
package (see ``calibration.py``); ``CostModel()`` keeps the reference defaults
so that a plain ``schedule(tree)`` reproduces the reference's plan.
"""
from __future__ import annotations

import ctypes
from collections import Counter
from dataclasses import asdict, dataclass
import itertools
from math import ceil

import numpy as np

from .tree import KVTree


@dataclass(frozen=True)
class Job:
    """``requests`` attend over physical KV ``tokens`` (reference schedule.py:7-10)."""
    requests: tuple[int, ...]
    tokens: tuple[int, ...]


def _runs(positions):
    """Maximal runs ``(start, length)`` of consecutive positions, in order."""
    n = len(positions)
    if n > 16 and positions[-1] - positions[0] + 1 == n and tuple(positions) == tuple(range(positions[0],
                                                                                            positions[0] + n)):
        return ((positions[0], n),)      # one run, compared at C speed
    runs = []
    start = None
    length = 0
    for p in positions:
        if start is not None and p == start + length:
            length += 1
        else:
            if start is not None:
                runs.append((start, length))
            start, length = p, 1
    if start is not None:
        runs.append((start, length))
    return tuple(runs)


def _concat(a, b):
    """Concatenate two run tuples, merging a contiguous seam."""
    if not a:
        return b
    if not b:
        return a
    last_start, last_len = a[-1]
    first_start, first_len = b[0]
    if first_start == last_start + last_len:
        return a[:-1] + ((last_start, last_len + first_len),) + b[1:]
    return a + b


def _expand(runs):
    if len(runs) == 1:
        start, length = runs[0]
        return tuple(range(start, start + length))
    return tuple(itertools.chain.from_iterable(range(start, start + length) for start, length in runs))


def physical_jobs(jobs):
    """Cut every job at discontinuities of its positions (reference schedule.py:13-26)."""
    result = []
    for job in jobs:
        tokens = job.tokens
        if tokens[-1] - tokens[0] + 1 == len(tokens):
            result.append(job)
            continue
        offset = 0
        for start, length in _runs(tokens):
            result.append(Job(job.requests, tokens[offset:offset + length]))
            offset += length
    return result


@dataclass
class CostModel:
    """Roofline constants in bytes/us and FLOP/us (reference schedule.py:29-39).

    ``cube_rows`` is the largest query-row count handled by the small-group
    kernel, ``max_query_rows`` the query-row tile of the large-group kernel and
    the per-job request cap, ``key_tile`` the small-group key tile (the large
    group uses ``key_tile // 2``), ``kv_split`` the longest KV segment per job.
    """
    bandwidth: float = 900_000.0
    cube_flops: float = 100_000_000.0
    task_us: float = 0.15
    merge_us: float = 0.03
    cube_rows: int = 16
    key_tile: int = 128
    kv_split: int = 512
    max_query_rows: int = 64

    def cost(self, requests, tokens, qheads, kvheads, dim):
        """Estimated microseconds of one physical job (reference schedule.py:41-52)."""
        if not requests or not tokens:
            return 0.0
        nreq = len(requests)
        rows = nreq * (qheads // kvheads)
        small = rows <= self.cube_rows
        row_tile = self.cube_rows if small else self.max_query_rows
        col_tile = self.key_tile if small else self.key_tile // 2
        qtiles = ceil(rows / row_tile)
        ktiles = ceil(len(tokens) / col_tile)
        # Integer byte/FLOP counts, divided in the same order as the
        # reference so that plans tie-break identically.
        flops = 4 * qtiles * row_tile * ktiles * col_tile * dim * kvheads
        reads = 4 * len(tokens) * dim * kvheads * qtiles
        partial = 4 * nreq * qheads * (dim + 1)
        return (max(flops / self.cube_flops, reads / self.bandwidth)
                + self.task_us * qtiles * kvheads
                + partial / self.bandwidth
                + self.merge_us * nreq)

    @classmethod
    def b200(cls):
        """Constants fitted to this package's sm_100a kernels on one B200.

        Fitted on the calibration grid in ``calibration.py`` (disjoint from the
        evaluation tree grid); the fit procedure is ``calibration.fit``.
        """
        from .calibration import B200_CONSTANTS
        return cls(**B200_CONSTANTS)


@dataclass
class Plan:
    """A schedule: jobs, method, estimated microseconds, settings (reference schedule.py:55-60)."""
    jobs: list[Job]
    method: str
    estimated_us: float
    settings: dict

    def validate(self, tree):
        """Raise ``ValueError`` unless the jobs cover each request's path exactly once."""
        covered = [Counter() for _ in tree.paths]
        for job in self.jobs:
            for request in job.requests:
                covered[request].update(job.tokens)
        for request, path in enumerate(tree.paths):
            if covered[request] != Counter(path):
                raise ValueError(f"Plan does not partition request {request}'s context")


def _chain_tuple(chain):
    """The children of a (last child, earlier chain) chain, first to last."""
    out = []
    while chain is not None:
        out.append(chain[0])
        chain = chain[1]
    return tuple(reversed(out))


class _Planner:
    """Memoised cost evaluation and the greedy / subset-DP recursions for one call."""

    def __init__(self, tree, qheads, kvheads, dim, model):
        self.nodes = tree.nodes
        self.node_runs = [_runs(n.tokens) for n in tree.nodes]
        self.node_size = [len(n.requests) for n in tree.nodes]
        self.qheads, self.kvheads, self.dim = qheads, kvheads, dim
        self.model = model
        self.req_tile = max(1, model.max_query_rows // (qheads // kvheads))
        self.kv_split = model.kv_split
        self.piece_memo = {}
        self.count_memo = {}
        self.pieces_memo = {}
        self.solve_memo = {}

    # -- costs -------------------------------------------------------------
    def piece_cost(self, nreq, ntok):
        key = (nreq, ntok)
        value = self.piece_memo.get(key)
        if value is None:
            value = self.model.cost(range(nreq), range(ntok), self.qheads, self.kvheads, self.dim)
            self.piece_memo[key] = value
        return value

    def chunk_pieces(self, runs):
        """Lengths of the physical jobs of every ``kv_split`` chunk, in order.

        A chunk is kept whole when ``last - first + 1 == len`` (the reference's
        contiguity test), otherwise it is cut into its maximal runs.
        """
        chunks = []
        current = []
        used = 0          # positions placed in the current chunk
        for start, length in runs:
            while length:
                take = min(length, self.kv_split - used)
                current.append((start, take))
                start += take
                used += take
                length -= take
                if used == self.kv_split:
                    chunks.append(current)
                    current, used = [], 0
        if current:
            chunks.append(current)
        pieces = []
        for chunk in chunks:
            total = sum(take for _, take in chunk)
            first = chunk[0][0]
            last = chunk[-1][0] + chunk[-1][1] - 1
            if last - first + 1 == total:
                pieces.append(total)
            else:
                pieces.extend(take for _, take in chunk)
        return pieces

    def count_cost(self, count, runs):
        """Cost of ``count`` requests attending over ``runs`` (reference ``count_cost``)."""
        key = (count, runs)
        value = self.count_memo.get(key)
        if value is None:
            pieces = self.pieces_memo.get(runs)
            if pieces is None:
                pieces = self.pieces_memo[runs] = self.chunk_pieces(runs)
            costs = []
            for q in range(0, count, self.req_tile):
                nreq = min(self.req_tile, count - q)
                costs.extend(self.piece_cost(nreq, take) for take in pieces)
            value = sum(costs)
            self.count_memo[key] = value
        return value

    # -- recursions --------------------------------------------------------
    def solve(self, method, node_id, inherited):
        key = (node_id, inherited)
        hit = self.solve_memo.get(key)
        if hit is not None:
            return hit
        node = self.nodes[node_id]
        runs = _concat(inherited, self.node_runs[node_id])
        if not node.children:
            result = (self.count_cost(self.node_size[node_id], runs), ())
        elif method == "greedy":
            result = self._solve_greedy(node, runs)
        else:
            result = self._solve_subsets(node, node_id, runs)
        self.solve_memo[key] = result
        return result

    def _solve_greedy(self, node, runs):
        remaining = len(node.requests)
        pushed = []
        for child in node.children:
            count = self.node_size[child]
            child_runs = self.node_runs[child]
            keep_apart = self.count_cost(remaining, runs) + self.count_cost(count, child_runs)
            push_down = (self.count_cost(remaining - count, runs)
                         + self.count_cost(count, _concat(runs, child_runs)))
            if push_down < keep_apart:
                pushed.append(child)
                remaining -= count
        total = self.count_cost(remaining, runs)
        total += sum(self.solve("greedy", child, runs if child in pushed else ())[0]
                     for child in node.children)
        return total, tuple(pushed)

    def _solve_subsets(self, node, node_id, runs):
        # states: detached-request count -> (best subtotal, pushed children),
        # the pushed children as a chain (last child, earlier chain) so that
        # extending a state costs O(1); tuples are built once at the end, where
        # ties between totals are broken by the pushed tuples as in the reference.
        states = {0: (0.0, None)}
        for child in node.children:
            count = self.node_size[child]
            apart = self.solve("cube", child, ())[0]
            together = self.solve("cube", child, runs)[0]
            updated = {}
            get = updated.get
            for removed, (subtotal, pushed) in states.items():
                value = subtotal + apart
                best = get(removed)
                if best is None or value < best[0]:
                    updated[removed] = (value, pushed)
                slot = removed + count
                value = subtotal + together
                best = get(slot)
                if best is None or value < best[0]:
                    updated[slot] = (value, (child, pushed))
            states = updated
        size = self.node_size[node_id]
        return min((subtotal + self.count_cost(size - removed, runs), _chain_tuple(pushed))
                   for removed, (subtotal, pushed) in states.items())

    # -- job materialisation -----------------------------------------------
    def split(self, requests, runs_or_tokens, runs=True):
        tokens = _expand(runs_or_tokens) if runs else tuple(runs_or_tokens)
        requests = tuple(requests)
        return [Job(requests[q:q + self.req_tile], tokens[k:k + self.kv_split])
                for q in range(0, len(requests), self.req_tile)
                for k in range(0, len(tokens), self.kv_split)]

    def native_pushed(self, method):
        """Per node, whether the plan pushes its parent's positions into it, by ``ta_schedule_tree``.

        The library runs the same recursion as ``solve`` (costs, sums and ties
        computed identically); None when the cost model is not this module's
        ``CostModel.cost`` (a subclass with its own formula runs ``solve``).
        """
        if type(self.model).cost is not CostModel.cost:
            return None
        from . import _lib
        lib = _lib.load()
        n = len(self.nodes)
        child_offsets = np.zeros(n + 1, dtype=np.int32)
        np.cumsum([len(node.children) for node in self.nodes], out=child_offsets[1:])
        children = np.fromiter(itertools.chain.from_iterable(node.children for node in self.nodes),
                               dtype=np.int32, count=int(child_offsets[-1]))
        sizes = np.array(self.node_size, dtype=np.int32)
        run_offsets = np.zeros(n + 1, dtype=np.int32)
        np.cumsum([len(r) for r in self.node_runs], out=run_offsets[1:])
        runs = np.fromiter(itertools.chain.from_iterable(p for r in self.node_runs for p in r), dtype=np.int64,
                           count=2 * int(run_offsets[-1]))
        m = self.model
        model = _lib.CostModelC(m.bandwidth, m.cube_flops, m.task_us, m.merge_us, m.cube_rows, m.key_tile,
                                m.kv_split, m.max_query_rows)
        pushed = np.zeros(n, dtype=np.uint8)
        rc = lib.ta_schedule_tree(child_offsets.ctypes.data, children.ctypes.data, sizes.ctypes.data,
                                  run_offsets.ctypes.data, runs.ctypes.data, n,
                                  _lib.SCHEDULE_CUBE if method == "cube" else _lib.SCHEDULE_GREEDY,
                                  ctypes.byref(model), self.qheads, self.kvheads, self.dim, pushed.ctypes.data,
                                  None)
        _lib.check(rc, "ta_schedule_tree")
        return pushed.tolist()

    def materialize(self, method, native=True):
        flags = self.native_pushed(method) if native else None
        jobs = []
        stack = [(0, ())]
        while stack:
            node_id, inherited = stack.pop()
            node = self.nodes[node_id]
            runs = _concat(inherited, self.node_runs[node_id])
            if flags is None:
                _, pushed = self.solve(method, node_id, inherited)
            else:
                pushed = tuple(c for c in node.children if flags[c])
            detached = {r for child in pushed for r in self.nodes[child].requests}
            remaining = tuple(r for r in node.requests if r not in detached)
            jobs.extend(self.split(remaining, runs))
            # Pre-order traversal: children in order, so push them reversed.
            for child in reversed(node.children):
                stack.append((child, runs if child in pushed else ()))
        return jobs

    def total_cost(self, jobs):
        return sum(self.model.cost(j.requests, j.tokens, self.qheads, self.kvheads, self.dim)
                   for j in physical_jobs(jobs))


def schedule(tree: KVTree, qheads=32, kvheads=8, dim=128, method="cube", model=None, _native=True):
    """Plan the jobs of ``tree`` with ``method`` in {request, fixed, greedy, cube}.

    The greedy and subset-DP decisions come from the library's native
    ``ta_schedule_tree``; ``_native=False`` runs the Python statement of the
    same recursion (``_Planner.solve``), which tests hold identical to it.
    """
    if qheads % kvheads:
        raise ValueError("Query heads must be divisible by KV heads")
    model = model or CostModel()
    planner = _Planner(tree, qheads, kvheads, dim, model)
    if method == "request":
        jobs = [j for r, path in enumerate(tree.paths) for j in planner.split((r,), path, runs=False)]
    elif method == "fixed":
        jobs = [j for n in tree.nodes for j in planner.split(n.requests, n.tokens, runs=False)]
    elif method in ("greedy", "cube"):
        jobs = planner.materialize(method, _native)
    else:
        raise ValueError(f"Unknown scheduling method: {method}")
    settings = asdict(model)
    settings.update(qheads=qheads, kvheads=kvheads, head_dim=dim)
    return Plan(jobs, method, planner.total_cost(jobs), settings)
