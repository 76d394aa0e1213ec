"""prepare(): reference metadata bit-exact, plus the consistency of the B200 arrays."""
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from tree_attention import CostModel, KVTree, schedule
from tree_attention import kernels
from tests.golden.make_golden import TREE_SPECS, build_tree

HERE = Path(__file__).parent / "golden"
PREP = np.load(HERE / "prepare.npz")
GOLDEN = json.loads((HERE / "plans.json").read_text())
SPECS = {s["name"]: s for s in TREE_SPECS}
KEYS = sorted({k.rsplit("|", 1)[0] for k in PREP.files})


class _Lib:
    KVTree = KVTree


@pytest.mark.parametrize("key", KEYS)
def test_prepare_matches_reference(key):
    name, model, qh, method = key.split("|")
    model, qh = int(model), int(qh)
    kh, d = (8, 128) if qh == 32 else (2, 32)
    tree = build_tree(_Lib, SPECS[name])
    plan = schedule(tree, qh, kh, d, method, CostModel(**GOLDEN["cost_models"][model]))
    p = kernels.prepare(plan, torch.empty(len(tree.paths), qh, d))
    order = np.array([x for j in p.jobs for x in (len(j.requests), j.tokens[0], len(j.tokens))] +
                     [r for j in p.jobs for r in j.requests], dtype=np.int64)
    np.testing.assert_array_equal(order, PREP[key + "|order"])
    for field in ("qids", "kids", "qlen", "klen", "slots", "counts"):
        got = getattr(p, field).numpy()
        assert got.dtype == np.int32
        np.testing.assert_array_equal(got, PREP[f"{key}|{field}"], err_msg=field)
    flags = PREP[key + "|flags"]
    assert [p.small_jobs, int(p.contiguous_k), int(p.contiguous_q)] == flags.tolist()
    check_b200_arrays(p, qh // kh)


def check_b200_arrays(p, groups, heads=None):
    meta = p.host_arrays
    heads = heads or p.num_kv_heads
    qlen, klen, qids = meta["qlen"], meta["klen"], meta["qids"]
    pieces, pcounts, cslots = meta["pieces"], meta["pcounts"], meta["cslots"]
    # pieces tile every job's keys in order, with consecutive partial slots
    slot = 0
    next_key = {}
    for job, offset, keys, first in pieces:
        job, offset, keys = int(job), int(offset), int(keys)
        assert offset == next_key.get(job, 0) and keys > 0
        next_key[job] = offset + keys
        assert first == slot
        slot += int(qlen[job])
    assert next_key == {j: int(klen[j]) for j in range(len(qlen))}
    assert meta["num_partials"] == slot
    # each request's partial slots: one per piece of every job it belongs to, in piece order
    for r in range(len(pcounts)):
        want = [int(first) + j for job, _, _, first in pieces for j in range(qlen[job]) if qids[job, j] == r]
        assert pcounts[r] == len(want)
        assert cslots[r, :pcounts[r]].tolist() == want
    # every (piece, row tile, head) is covered exactly once by the task lists
    covered = {}
    for piece, tile in meta["small_tasks"]:
        key = (int(piece), "s", int(tile))
        covered[key] = covered.get(key, 0) + 1
    for piece, pair, q0, _ in meta["tc_tasks"]:
        key = (int(piece), "t", int(pair))
        covered[key] = covered.get(key, 0) + 1
        job = int(pieces[piece][0])
        reqs = qids[job, :qlen[job]].tolist()
        assert q0 == (reqs[0] if reqs == list(range(reqs[0], reqs[0] + len(reqs))) else -1)
    slot_piece = {int(first): pc for pc, (_, _, _, first) in enumerate(pieces)}
    segs = meta["kn_segs"]
    for first, nseg, _, _ in meta["kn_tasks"]:
        assert 1 <= nseg <= kernels.KN_PACK_SEGS
        row0 = kt = 0
        for head, r0, rows, prow, k0, seg_kt, keys, jobf, q0, qofs, _, _ in segs[first:first + nseg]:
            job, growing = int(jobf) & 0x3FFFFFFF, int(jobf) >> 30
            assert prow % groups == 0 and rows % groups == 0 and qofs * groups + rows <= qlen[job] * groups
            pc = slot_piece[int(prow) // groups - int(qofs)]
            assert pieces[pc, 0] == job and keys == pieces[pc, 2]
            assert rows == min(max(groups, kernels.KN_TASK_ROWS // groups * groups), qlen[job] * groups - qofs * groups)
            assert k0 == p.jobs[job].tokens[0] + pieces[pc, 1] and growing in (0, 1)
            reqs = p.jobs[job].requests
            assert q0 == (reqs[0] + qofs if reqs[-1] - reqs[0] + 1 == len(reqs) else -1)
            assert r0 == row0 and (nseg == 1 and seg_kt == 0 or seg_kt == kt)
            if nseg > 1:
                assert keys <= kernels.KEY_TILE
            row0 += rows
            kt += -(-int(keys) // kernels.KN_BOX) * kernels.KN_BOX
            key = (pc, "k", int(head), int(qofs))
            covered[key] = covered.get(key, 0) + 1
        if nseg > 1:
            assert kt <= kernels.KEY_TILE and row0 <= kernels.KN_PACK_ROWS
    assert all(v == 1 for v in covered.values())
    rows_covered = np.zeros(len(pieces), dtype=np.int64)
    for (piece, kind, idx, *sub) in covered:
        rows = int(qlen[pieces[piece, 0]]) * groups
        if kind == "k":
            chunk = max(groups, kernels.KN_TASK_ROWS // groups * groups)
            assert rows <= kernels.KN_ROWS and all((piece, "k", h, sub[0]) in covered for h in range(heads))
            if idx == 0:
                rows_covered[piece] += min(chunk, rows - sub[0] * groups)
        else:
            size = kernels.SMALL_ROWS if kind == "s" else kernels.TC_ROWS
            if kind == "t":
                assert rows > kernels.KN_ROWS
            rows_covered[piece] += min(size, rows - idx * size)
    want_rows = qlen[pieces[:, 0]].astype(np.int64) * groups
    np.testing.assert_array_equal(rows_covered, want_rows)
    # small tasks are grouped by padded row class 4 / 8 / 16
    end = meta["small_class_end"]
    for idx, (piece, tile) in enumerate(meta["small_tasks"]):
        rows = min(kernels.SMALL_ROWS, qlen[pieces[piece, 0]] * groups - tile * kernels.SMALL_ROWS)
        cls = 0 if idx < end[0] else (1 if idx < end[1] else 2)
        assert rows <= (4, 8, 16)[cls]
    L = p.layout
    # persistent CTA lists partition the keys-in-lanes tasks
    offs = meta["kn_offsets"]
    assert offs[0] == 0 and offs[-1] == len(meta["kn_tasks"]) and np.all(np.diff(offs) >= 0)
    assert len(offs) == meta["kn_ctas"] + 1
    # CTAs of each row class hold only tasks of that class, classes in order
    cc = meta["kn_class_ctas"]
    assert int(cc.sum()) == meta["kn_ctas"]
    assert [L.kn_class_ctas[c] for c in range(5)] == cc.tolist()
    cta = 0
    for c, n in enumerate(cc.tolist()):
        for b in range(cta, cta + n):
            assert offs[b + 1] > offs[b]                  # no idle CTA
            for f, nseg, _, _ in meta["kn_tasks"][offs[b]:offs[b + 1]]:
                assert kernels.kn_class(int(segs[f:f + nseg, 2].sum())) == c
        cta += n
    assert all(getattr(L, "off_" + name) % 4 == 0 for name in ("pieces", "cslots", "kn_tasks", "kn_segs", "kn_offsets"))
    # layout offsets address the same arrays as the views
    flat = p.metadata.numpy()
    L = p.layout
    np.testing.assert_array_equal(flat[L.off_qids:L.off_qids + qids.size], qids.ravel())
    np.testing.assert_array_equal(flat[L.off_cslots:L.off_cslots + cslots.size], cslots.ravel())
    np.testing.assert_array_equal(flat[L.off_pieces:L.off_pieces + pieces.size], pieces.ravel())
    np.testing.assert_array_equal(flat[L.off_kn_tasks:L.off_kn_tasks + meta["kn_tasks"].size], meta["kn_tasks"].ravel())
    np.testing.assert_array_equal(flat[L.off_kn_segs:L.off_kn_segs + segs.size], segs.ravel())
    assert L.num_jobs == len(qlen) and L.max_requests == qids.shape[1] and L.num_requests == len(pcounts)
    assert L.num_pieces == len(pieces) and L.max_pslots == cslots.shape[1]


@pytest.mark.parametrize("use_tc", [False, True])
def test_task_lists_cover_rows(use_tc, monkeypatch):
    monkeypatch.setattr(kernels, "tc_supported", lambda d, dt: use_tc)
    tree = KVTree.synthetic([-1] + [0] * 128, [8128] + [64] * 128, list(range(1, 129)))
    for model in (CostModel(), CostModel.b200()):
        for method in ("request", "fixed", "cube"):
            p = kernels.prepare(schedule(tree, method=method, model=model), torch.empty(128, 32, 128))
            check_b200_arrays(p, 4)
            meta = p.host_arrays
            if use_tc:
                assert len(meta["small_tasks"]) == 0
                assert all(meta["qlen"][meta["pieces"][pc, 0]] * 4 > kernels.KN_ROWS for pc, _, _, _ in meta["tc_tasks"])
            else:
                assert len(meta["tc_tasks"]) == 0 and len(meta["kn_tasks"]) == 0


def test_cached_decode_plan_tails():
    tree = KVTree.synthetic([-1, 0, 0], [64, 16, 16], [1, 2])
    plan = schedule(tree, method="cube")
    q = torch.empty(2, 32, 128)
    # host-side construction only: the tail jobs and their indices
    tails = [kernels.Job((r,), tuple(range(96 + r * 8, 96 + (r + 1) * 8))) for r in range(2)]
    p = kernels.prepare(kernels.Plan(plan.jobs + tails, plan.method, plan.estimated_us, plan.settings), q)
    tail_ids = [i for i, j in enumerate(p.jobs) if j.tokens[0] >= 96]
    assert len(tail_ids) == 2 and all(p.qlen[i] == 1 and p.klen[i] == 8 for i in tail_ids)


def test_prepare_rejects_bad_plans():
    tree = KVTree.from_sequences([[1, 2], [1, 3]])
    plan = schedule(tree, 8, 2, 32)
    with pytest.raises(ValueError):
        kernels.prepare(plan, torch.empty(1, 8, 32))   # request 1 outside a batch of 1
    with pytest.raises(ValueError):
        kernels.prepare(plan, torch.empty(2, 6, 32), num_kv_heads=4)


def test_pieces_split_long_jobs_and_keep_tails_whole():
    # one job of 4 requests (16 rows) over 8192 keys: keys-in-lanes, cut into pieces
    tree = KVTree.synthetic([-1] + [0] * 4, [8192] + [32] * 4, list(range(1, 5)))
    plan = schedule(tree, method="fixed", model=CostModel(kv_split=1 << 20, max_query_rows=4096))
    q = torch.empty(4, 32, 128, dtype=torch.bfloat16)
    p = kernels.prepare(plan, q)
    meta = p.host_arrays
    assert sum(1 for j in p.jobs if len(j.requests) == 4) == 1
    root = [pc for pc in meta["pieces"] if meta["qlen"][pc[0]] == 4]
    assert len(root) > 1 and sum(int(pc[2]) for pc in root) == 8192
    assert all(pc[2] % kernels.KEY_TILE == 0 for pc in root[:-1])
    chunk = kernels.KN_TASK_ROWS
    assert len(meta["kn_segs"]) == sum(8 * -(-int(meta["qlen"][pc[0]]) * 4 // chunk) for pc in meta["pieces"])
    check_b200_arrays(p, 4)
    # decode tails (positions past the prompt) are never split and follow klen
    tails = [kernels.Job((r,), tuple(range(tree.storage_tokens + r * 4096, tree.storage_tokens + (r + 1) * 4096)))
             for r in range(4)]
    p2 = kernels.prepare(kernels.Plan(plan.jobs + tails, plan.method, plan.estimated_us, plan.settings), q,
                         _no_split_from=tree.storage_tokens)
    m2 = p2.host_arrays
    tail_jobs = [i for i, j in enumerate(p2.jobs) if j.tokens[0] >= tree.storage_tokens]
    for i in tail_jobs:
        assert sum(1 for pc in m2["pieces"] if pc[0] == i) == 1
    flags = {int(rec[7]) & 0x3FFFFFFF: int(rec[7]) >> 30 for rec in m2["kn_segs"]}
    assert all(flags[i] == 1 for i in tail_jobs) and all(f == 0 for j, f in flags.items() if j not in tail_jobs)
    check_b200_arrays(p2, 4)


def test_lpt_assignment_balances():
    costs = [9, 1, 1, 1, 5, 5, 4, 3, 3, 2]
    offsets, order = kernels.assign_lpt(costs, 3)
    loads = [sum(costs[t] for t in order[offsets[b]:offsets[b + 1]]) for b in range(3)]
    assert sorted(order.tolist()) == list(range(len(costs)))
    assert max(loads) == 12 and sum(loads) == sum(costs)


def test_packing_shares_tiles_between_short_segments():
    # 128 private 64-key leaves x 8 heads: two leaves per 128-key tile
    tree = KVTree.synthetic([-1] + [0] * 128, [8128] + [64] * 128, list(range(1, 129)))
    p = kernels.prepare(schedule(tree, method="cube", model=CostModel.b200()), torch.empty(128, 32, 128, dtype=torch.bfloat16))
    meta = p.host_arrays
    counts = [int(n) for _, n, _, _ in meta["kn_tasks"]]
    assert sum(counts) == len(meta["kn_segs"]) and max(counts) == 2 and counts.count(2) == 512
    assert p.layout.kn_class_ctas[1] > 0 and sum(p.layout.kn_class_ctas[c] for c in (0, 2, 3, 4)) == 0
    check_b200_arrays(p, 4)
    # mixed spans and rows never exceed a tile
    items = [(h, 4 * (1 + (i % 2)), i, 1000 * i, 1 + (i * 37) % 200, i, -1, 0) for i in range(60) for h in range(2)]
    for task in kernels.pack_segments(items):
        if len(task) > 1:
            assert sum(-(-it[4] // 32) * 32 for it in task) <= 128 and sum(it[1] for it in task) <= 16
            assert len(task) <= kernels.KN_PACK_SEGS
    assert sorted(it for task in kernels.pack_segments(items) for it in task) == sorted(items)
