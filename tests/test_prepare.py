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


def check_b200_arrays(p, groups):
    meta = p.host_arrays
    qlen, slots, cslots, counts = meta["qlen"], meta["slots"], meta["cslots"], meta["counts"]
    maxr = meta["qids"].shape[1]
    base = meta["slot_base"]
    assert base[0] == 0 and np.all(np.diff(base) == qlen[:-1])
    assert meta["num_partials"] == qlen.sum()
    for r in range(len(counts)):
        for k in range(counts[r]):
            job, j = divmod(int(slots[r, k]), maxr)
            assert cslots[r, k] == base[job] + j
            assert meta["qids"][job, j] == r
    # every (job, row tile) is covered exactly once by the task lists
    covered = {}
    for job, tile in meta["small_tasks"]:
        covered[(int(job), int(tile), "s")] = covered.get((int(job), int(tile), "s"), 0) + 1
    for job, tile in meta["tc_tasks"]:
        covered[(int(job), int(tile), "t")] = covered.get((int(job), int(tile), "t"), 0) + 1
    assert all(v == 1 for v in covered.values())
    rows_covered = np.zeros(len(qlen), dtype=np.int64)
    for (job, tile, kind) in covered:
        size = kernels.SMALL_ROWS if kind == "s" else kernels.TC_ROWS
        rows_covered[job] += min(size, qlen[job] * groups - tile * size)
    np.testing.assert_array_equal(rows_covered, qlen.astype(np.int64) * groups)
    # small tasks are grouped by padded row class 4 / 8 / 16
    end = meta["small_class_end"]
    for idx, (job, tile) in enumerate(meta["small_tasks"]):
        rows = min(kernels.SMALL_ROWS, qlen[job] * groups - tile * kernels.SMALL_ROWS)
        cls = 0 if idx < end[0] else (1 if idx < end[1] else 2)
        assert rows <= (4, 8, 16)[cls]
    # layout offsets address the same arrays as the views
    flat = p.metadata.numpy()
    L = p.layout
    np.testing.assert_array_equal(flat[L.off_qids:L.off_qids + meta["qids"].size], meta["qids"].ravel())
    np.testing.assert_array_equal(flat[L.off_cslots:L.off_cslots + cslots.size], cslots.ravel())
    assert L.num_jobs == len(qlen) and L.max_requests == maxr and L.num_requests == len(counts)


@pytest.mark.parametrize("use_tc", [False, True])
def test_task_lists_cover_rows(use_tc, monkeypatch):
    monkeypatch.setattr(kernels, "tc_supported", lambda d, dt: use_tc)
    tree = KVTree.synthetic([-1] + [0] * 128, [8128] + [64] * 128, list(range(1, 129)))
    for model in (CostModel(), CostModel.b200()):
        for method in ("request", "fixed", "cube"):
            p = kernels.prepare(schedule(tree, method=method, model=model), torch.empty(128, 32, 128))
            check_b200_arrays(p, 4)
            if use_tc:
                assert all(p.host_arrays["qlen"][j] * 4 > 16 for j, _ in p.host_arrays["tc_tasks"])


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
