"""Scheduler plans vs the reference's plans, plus the reference's semantic tests."""
import gc
import json
import weakref
from pathlib import Path

import pytest

from tree_attention import CostModel, KVTree, schedule
from tree_attention.schedule import Plan, physical_jobs
from tests.golden.make_golden import TREE_SPECS, build_tree, plan_digest, runs

GOLDEN = json.loads((Path(__file__).parent / "golden" / "plans.json").read_text())
SPECS = {s["name"]: s for s in TREE_SPECS}


class _Lib:
    KVTree = KVTree


_TREES = {}


def tree_named(name):
    if name not in _TREES:
        _TREES[name] = build_tree(_Lib, SPECS[name])
    return _TREES[name]


def check_plan(plan, expected):
    assert plan.method == expected["method"]
    assert len(plan.jobs) == expected["njobs"]
    assert float(plan.estimated_us).hex() == expected["estimated_us"]
    assert plan_digest(plan.jobs) == expected["digest"]
    assert plan.settings == expected["settings"]
    if "jobs" in expected:
        assert [[list(j.requests), runs(j.tokens)] for j in plan.jobs] == expected["jobs"]


@pytest.mark.parametrize("row", GOLDEN["plans"],
                         ids=[f"{r['tree']}-m{r['model']}-{r['heads'][0]}-{r['method']}" for r in GOLDEN["plans"]])
def test_plan_bit_exact(row):
    qh, kh, d = row["heads"]
    model = CostModel(**GOLDEN["cost_models"][row["model"]])
    plan = schedule(tree_named(row["tree"]), qh, kh, d, row["method"], model)
    check_plan(plan, row["plan"])


def test_tree_scan_bit_exact():
    """The 81-tree scan of the reference's scripts/scan_trees.py:7-15."""
    for row in GOLDEN["scan"]:
        tree = KVTree.synthetic([-1, 0, 0, 1, 1, 2, 2], row["lengths"], [3, 4, 5, 6])
        for method in ("request", "fixed", "greedy", "cube"):
            plan = schedule(tree, method=method)
            assert [float(plan.estimated_us).hex(), len(plan.jobs)] == row[method], (row["lengths"], method)


def test_reference_evaluation_grid_bit_exact():
    """All 81 trees x 4 methods of the reference's scripts/tree_shapes.py grid."""
    for row in GOLDEN["reference_grid"]:
        tree = KVTree.synthetic(*row["synthetic"])
        for method in ("request", "fixed", "greedy", "cube"):
            check_plan(schedule(tree, method=method), row[method])


def test_dynamic_plan_minimizes_global_estimated_cost():
    # reference tests/test_semantics.py:45-54
    for root in (16, 128, 1024):
        for child in (8, 64, 256):
            for leaf in (16, 128, 512):
                tree = KVTree.synthetic([-1, 0, 0, 1, 1, 2, 2], [root, child, child, leaf, 2 * leaf, leaf, 2 * leaf],
                                        [3, 4, 5, 6])
                greedy = schedule(tree, method="greedy")
                dynamic = schedule(tree, method="cube")
                dynamic.validate(tree)
                assert dynamic.estimated_us <= greedy.estimated_us + 1e-10


def test_schedule_releases_input_tree():
    # reference tests/test_semantics.py:56-67
    gc.disable()
    try:
        for method in ("request", "fixed", "greedy", "cube"):
            tree = KVTree.from_sequences([[1, 2, 3], [1, 2, 4]])
            ref = weakref.ref(tree)
            plan = schedule(tree, method=method)
            del tree
            assert ref() is None, method
            assert plan.jobs
    finally:
        gc.enable()


def test_plan_detects_double_counting():
    # reference tests/test_semantics.py:69-74
    tree = KVTree.from_sequences([[1, 2], [1, 3]])
    plan = schedule(tree)
    plan.jobs.append(plan.jobs[0])
    with pytest.raises(ValueError):
        plan.validate(tree)


@pytest.mark.parametrize("name", sorted(SPECS))
def test_every_plan_partitions_contexts(name):
    tree = tree_named(name)
    for method in ("request", "fixed", "greedy", "cube"):
        for model in (CostModel(), CostModel(kv_split=48), CostModel.b200()):
            plan = schedule(tree, 32, 8, 128, method, model)
            plan.validate(tree)
            Plan(physical_jobs(plan.jobs), method, plan.estimated_us, plan.settings).validate(tree)


def test_errors():
    tree = KVTree.from_sequences([[1, 2]])
    with pytest.raises(ValueError):
        schedule(tree, 6, 4)
    with pytest.raises(ValueError):
        schedule(tree, method="bogus")


def test_physical_jobs_cuts_discontinuities():
    from tree_attention.schedule import Job
    jobs = physical_jobs([Job((0,), (0, 1, 2, 5, 6, 9)), Job((1,), (3, 4))])
    assert [(j.requests, j.tokens) for j in jobs] == [((0,), (0, 1, 2)), ((0,), (5, 6)), ((0,), (9,)),
                                                      ((1,), (3, 4))]


def test_reference_headline_plan_fixture():
    """bench.py's reference arm times the oracle on the reference's own headline plan (headline_plan.json):
    the fixture is that plan job by job, the same plan plans.json pins by digest, and the same plan this
    package's scheduler produces with the reference's default cost model."""
    recorded = json.loads((Path(__file__).parent / "golden" / "headline_plan.json").read_text())
    assert plan_digest_of_runs(recorded["jobs"]) == recorded["digest"]
    row = next(r for r in GOLDEN["plans"] if r["tree"] == "headline" and r["model"] == 0
               and r["heads"] == [32, 8, 128] and r["method"] == "cube")
    assert recorded["digest"] == row["plan"]["digest"] and recorded["njobs"] == row["plan"]["njobs"]
    plan = schedule(tree_named("headline"), 32, 8, 128, "cube", CostModel())
    assert [[list(j.requests), runs(j.tokens)] for j in plan.jobs] == recorded["jobs"]


def plan_digest_of_runs(jobs):
    import hashlib
    canon = json.dumps(jobs, separators=(",", ":"))
    return hashlib.sha256(canon.encode()).hexdigest()
