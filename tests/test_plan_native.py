"""The native host planners against their Python statements, bit for bit.

* ``ta_plan_build`` (csrc/plan.cpp) against ``build_metadata`` +
  ``flatten_metadata``: ``prepare`` uploads the native builder's buffer.
* ``ta_schedule_tree`` (csrc/schedule.cpp) against ``_Planner.solve``:
  ``schedule`` takes its greedy / subset-DP decisions from the library.

Both run on the host, so these tests need no GPU.
"""
import ctypes
import random

import numpy as np
import pytest
import torch

from tree_attention import CostModel, KVTree, schedule
from tree_attention import _lib, kernels
from tree_attention.schedule import Job, physical_jobs
from tests.golden.make_golden import COST_MODELS, HEADS, METHODS, TREE_SPECS, build_tree


class _Lib:
    KVTree = KVTree


def layout_dict(layout):
    out = {}
    for name, _ in layout._fields_:
        value = getattr(layout, name)
        out[name] = list(value) if not isinstance(value, int) else value
    return out


def assert_native_matches(jobs, nreq, groups, use_tc, heads, sms, no_split_from=None):
    meta = kernels.build_metadata(jobs, nreq, groups, use_tc, heads, sms, no_split_from)
    flat, layout = kernels.flatten_metadata(meta, nreq)
    nflat, nlayout, nmeta = kernels._native_metadata(jobs, nreq, groups, use_tc, heads, sms, no_split_from)
    assert layout_dict(nlayout) == layout_dict(layout)
    assert nflat.dtype == np.int32
    np.testing.assert_array_equal(nflat, flat)
    for name in kernels._ORDER:
        assert nmeta[name].shape == meta[name].shape, name
        np.testing.assert_array_equal(nmeta[name], meta[name], err_msg=name)
    for name in ("small_max_keys", "kn_ctas", "num_partials", "contiguous_k"):
        assert nmeta[name] == meta[name], name
    for name in ("small_class_end", "kn_class_ctas"):
        np.testing.assert_array_equal(nmeta[name], meta[name], err_msg=name)


def sorted_jobs(plan, groups):
    jobs = physical_jobs(plan.jobs)
    jobs.sort(key=lambda job: len(job.requests) * groups > 16)
    return jobs


CASES = [(spec["name"], m, h, method) for spec in TREE_SPECS for m in range(len(COST_MODELS))
         for h in range(len(HEADS)) for method in METHODS
         if not (spec["name"] == "headline" and method == "request")]


@pytest.mark.parametrize("name,model,heads,method", CASES)
def test_native_builder_matches_on_reference_trees(name, model, heads, method):
    spec = next(s for s in TREE_SPECS if s["name"] == name)
    qh, kh, d = HEADS[heads]
    tree = build_tree(_Lib, spec)
    plan = schedule(tree, qh, kh, d, method, CostModel(**COST_MODELS[model]))
    groups = qh // kh
    jobs = sorted_jobs(plan, groups)
    nreq = len(tree.paths)
    assert_native_matches(jobs, nreq, groups, d == 128, kh, 148)
    # fewer SMs change the piece split and the CTA balance; the SIMT routes
    assert_native_matches(jobs, nreq, groups, d == 128, kh, 5)
    assert_native_matches(jobs, nreq, groups, False, kh, 148)


def test_native_builder_matches_on_headline_plans():
    tree = build_tree(_Lib, next(s for s in TREE_SPECS if s["name"] == "headline"))
    for method in ("request", "cube"):
        plan = schedule(tree, 32, 8, 128, method, CostModel.b200())
        jobs = sorted_jobs(plan, 4)
        for sms in (148, 132, 16):
            assert_native_matches(jobs, 128, 4, True, 8, sms)
        assert_native_matches(jobs, 128, 4, True, 4, 148)   # a two-GPU KV-head shard
        for heads in (2, 1):                                   # four- and eight-GPU shards
            assert_native_matches(jobs, 128, 4, True, heads, 148)


def test_query_tile_cut_level_follows_the_step_model():
    """The headline cube plan on one GPU keeps the widest cut (16 jobs x 8 heads = 128 query-tile CTAs,
    keys-in-lanes after them on 296 CTAs); a four-GPU shard (2 KV heads) stops one level earlier (96 CTAs
    of 3 tiles) and places the 128 keys-in-lanes tasks on the 104 CTAs the 52 free SMs hold."""
    tree = build_tree(_Lib, next(s for s in TREE_SPECS if s["name"] == "headline"))
    jobs = sorted_jobs(schedule(tree, 32, 8, 128, "cube", CostModel.b200()), 4)
    for heads, tc_ctas, kn_ctas in ((8, 128, 296), (4, 128, 256), (2, 96, 104), (1, 64, 64)):
        meta = kernels.build_metadata(jobs, 128, 4, True, heads=heads, sms=148)
        assert (len(meta["tc_tasks"]) * heads, int(meta["kn_ctas"])) == (tc_ctas, kn_ctas), heads
    levels = [(32, 8), (64, 4), (96, 3), (128, 2)]
    assert kernels.choose_tc_level(levels, [0, 128, 0, 0, 0], 148) == (96, 96)
    assert kernels.choose_tc_level([(128, 8)], [0, 512, 0, 0, 0], 148) == (None, None)
    assert kernels.choose_tc_level([], [0, 512, 0, 0, 0], 148) == (None, None)


def test_native_builder_matches_with_decode_tails():
    tree = build_tree(_Lib, next(s for s in TREE_SPECS if s["name"] == "decode_tree"))
    plan = schedule(tree, 32, 8, 128, "cube", CostModel.b200())
    prefix, nreq = tree.storage_tokens, len(tree.paths)
    for steps in (1, 16, 4096):
        tails = [Job((r,), tuple(range(prefix + r * steps, prefix + (r + 1) * steps))) for r in range(nreq)]
        jobs = physical_jobs(plan.jobs + tails)
        jobs.sort(key=lambda job: len(job.requests) * 4 > 16)
        for no_split in (None, prefix, 0):
            assert_native_matches(jobs, nreq, 4, True, 8, 148, no_split)


def random_jobs(rng, nreq):
    jobs = []
    for _ in range(rng.randint(1, 40)):
        size = rng.choice([1, 1, 2, 3, 4, 5, 8, rng.randint(1, nreq)])
        size = min(size, nreq)
        if rng.random() < 0.5:
            start = rng.randint(0, nreq - size)
            requests = tuple(range(start, start + size))
        else:
            requests = tuple(sorted(rng.sample(range(nreq), size)))
        keys = rng.choice([1, 7, 31, 32, 33, 64, 65, 96, 127, 128, 129, 256, 1000, rng.randint(1, 9000)])
        start = rng.randint(0, 50000)
        jobs.append(Job(requests, tuple(range(start, start + keys))))
    return jobs


def test_native_builder_matches_on_random_job_lists():
    rng = random.Random(20261202)
    for case in range(400):
        nreq = rng.randint(1, 96)
        groups = rng.choice([1, 2, 4, 8, 16])
        heads = rng.choice([1, 2, 4, 8])
        jobs = random_jobs(rng, nreq)
        jobs.sort(key=lambda job: len(job.requests) * groups > 16)
        no_split = rng.choice([None, None, 0, rng.randint(0, 50000)])
        sms = rng.choice([1, 2, 7, 148])
        assert_native_matches(jobs, nreq, groups, rng.random() < 0.8, heads, sms, no_split)


def test_prepare_uses_the_native_buffer():
    tree = build_tree(_Lib, next(s for s in TREE_SPECS if s["name"] == "small_config1"))
    plan = schedule(tree, 32, 8, 128, "cube", CostModel.b200())
    p = kernels.prepare(plan, torch.empty(len(tree.paths), 32, 128, dtype=torch.bfloat16))
    meta = kernels.build_metadata(p.jobs, len(tree.paths), 4, True, 8, kernels._sm_count(torch.device("cpu")))
    flat, layout = kernels.flatten_metadata(meta, len(tree.paths))
    np.testing.assert_array_equal(p.metadata.numpy(), flat)
    assert layout_dict(p.layout) == layout_dict(layout)


def test_plan_build_rejects_bad_arguments():
    lib = _lib.load()
    offs = np.array([0, 2], dtype=np.int32)
    reqs = np.array([0, 1], dtype=np.int32)
    k0 = np.array([0], dtype=np.int32)
    keys = np.array([100], dtype=np.int32)
    size = ctypes.c_int64(-1)
    layout = _lib.PlanLayout()

    def call(nreq=2, offs=offs, reqs=reqs, keys=keys, num_jobs=1, groups=4, capacity=0, meta=None):
        return lib.ta_plan_build(offs.ctypes.data, reqs.ctypes.data, k0.ctypes.data, keys.ctypes.data, num_jobs,
                                 nreq, groups, 1, 8, 148, -1, meta, capacity, ctypes.byref(size),
                                 ctypes.byref(layout))

    # too small a buffer: the size and layout are reported, nothing written
    assert call() == _lib.ERR_TOO_LARGE and size.value > 0 and layout.num_jobs == 1
    buf = np.full(size.value, -7, dtype=np.int32)
    assert call(capacity=size.value, meta=buf.ctypes.data) == 0
    assert buf[layout.off_qids:layout.off_qids + 2].tolist() == [0, 1]
    assert call(nreq=1) == _lib.ERR_ARG                                  # request 1 outside a batch of 1
    assert call(num_jobs=0) == _lib.ERR_ARG
    assert call(groups=0) == _lib.ERR_ARG
    assert call(keys=np.array([0], dtype=np.int32)) == _lib.ERR_ARG    # empty job
    assert call(offs=np.array([0, 0], dtype=np.int32)) == _lib.ERR_ARG  # job without requests
    assert lib.ta_plan_build(None, None, None, None, 1, 1, 1, 1, 1, 1, -1, None, 0, None, None) == _lib.ERR_ARG


# ---- the native scheduler (ta_schedule_tree, csrc/schedule.cpp) against _Planner.solve ----

def random_tree(rng):
    """A random radix tree: random branching, node lengths (some zero-length roots) and terminals."""
    n = rng.randint(2, 40)
    parents, lengths = [-1], [rng.choice([0, rng.randint(1, 3000)])]
    for i in range(1, n):
        parents.append(rng.randint(max(0, i - rng.choice([1, 3, i])), i - 1))
        lengths.append(rng.choice([1, 8, 31, 64, 129, rng.randint(1, 1200)]))
    has_child = set(parents[1:])
    terminals = [i for i in range(n) if i not in has_child]
    terminals += [i for i in range(1, n) if i in has_child and rng.random() < 0.2]
    rng.shuffle(terminals)
    return KVTree.synthetic(parents, lengths, terminals)


def random_model(rng):
    return CostModel(bandwidth=rng.choice([900_000.0, 6_000_000.0, 6.5e6 * rng.random() + 1e5]),
                     cube_flops=rng.choice([1e8, 1.2e9, 1.5e9 * rng.random() + 1e7]),
                     task_us=rng.choice([0.15, 0.02, rng.random()]), merge_us=rng.choice([0.03, 0.002, 0.0]),
                     cube_rows=rng.choice([4, 16, 32]), key_tile=rng.choice([64, 128, 256]),
                     kv_split=rng.choice([48, 100, 512, 2048, 1 << 20]),
                     max_query_rows=rng.choice([16, 64, 256, 512]))


def assert_same_plan(tree, qh, kh, d, method, model):
    native = schedule(tree, qh, kh, d, method, model)
    spec = schedule(tree, qh, kh, d, method, model, _native=False)
    assert native.jobs == spec.jobs
    assert native.estimated_us == spec.estimated_us


@pytest.mark.parametrize("method", ["greedy", "cube"])
def test_native_scheduler_matches_on_random_trees(method):
    rng = random.Random(7 if method == "cube" else 8)
    for _ in range(150):
        tree = random_tree(rng)
        qh, kh, d = rng.choice([(32, 8, 128), (8, 2, 32), (16, 16, 64), (64, 4, 128)])
        assert_same_plan(tree, qh, kh, d, method, random_model(rng))


def test_native_scheduler_matches_on_bench_trees():
    for name in ("headline", "decode_tree", "deep_bench", "wide", "no_share_root0"):
        tree = build_tree(_Lib, next(s for s in TREE_SPECS if s["name"] == name))
        for model in (CostModel(), CostModel.b200()):
            for method in ("greedy", "cube"):
                assert_same_plan(tree, 32, 8, 128, method, model)
    # a decode tree grown one token per leaf and step (non-contiguous leaf runs)
    tree = build_tree(_Lib, next(s for s in TREE_SPECS if s["name"] == "decode_tree"))
    prefix, nreq = tree.storage_tokens, len(tree.paths)
    leaves = list(range(len(tree.nodes) - nreq, len(tree.nodes)))
    for step in range(3):
        tree.extend_leaves(leaves, [prefix + r * 3 + step for r in range(nreq)])
        assert_same_plan(tree, 32, 8, 128, "cube", CostModel.b200())


def test_custom_cost_model_runs_the_python_recursion():
    class Flat(CostModel):
        def cost(self, requests, tokens, qheads, kvheads, dim):
            return 1.0 if requests and tokens else 0.0

    tree = build_tree(_Lib, next(s for s in TREE_SPECS if s["name"] == "deep_bench"))
    plan = schedule(tree, 32, 8, 128, "cube", Flat())
    assert plan.jobs == schedule(tree, 32, 8, 128, "cube", Flat(), _native=False).jobs
    plan.validate(tree)


def test_schedule_tree_rejects_bad_trees():
    lib = _lib.load()
    model = _lib.CostModelC(900_000.0, 1e8, 0.15, 0.03, 16, 128, 512, 64)
    offs = np.array([0, 1, 1], dtype=np.int32)
    kids = np.array([1], dtype=np.int32)
    sizes = np.array([2, 1], dtype=np.int32)
    roffs = np.array([0, 1, 2], dtype=np.int32)
    runs = np.array([0, 10, 10, 5], dtype=np.int64)
    pushed = np.full(2, 9, dtype=np.uint8)
    cost = ctypes.c_double(0.0)

    def call(kids=kids, runs=runs, method=_lib.SCHEDULE_CUBE, qh=32):
        return lib.ta_schedule_tree(offs.ctypes.data, kids.ctypes.data, sizes.ctypes.data, roffs.ctypes.data,
                                    runs.ctypes.data, 2, method, ctypes.byref(model), qh, 8, 128,
                                    pushed.ctypes.data, ctypes.byref(cost))

    assert call() == 0 and pushed.tolist() in ([0, 0], [0, 1]) and cost.value > 0
    assert call(kids=np.array([0], dtype=np.int32)) == _lib.ERR_ARG          # a node its own child
    assert call(runs=np.array([0, 10, 10, 0], dtype=np.int64)) == _lib.ERR_ARG  # an empty run
    assert call(method=3) == _lib.ERR_ARG
    assert call(qh=12) == _lib.ERR_ARG                                      # 12 query heads over 8 KV heads


def test_schedule_tree_bounds_its_depth():
    """The native recursion follows the tree's depth on the caller's stack: a chain of 2000 levels
    plans, a deeper one is rejected with an error code (no stack overflow)."""
    lib = _lib.load()
    model = _lib.CostModelC(900_000.0, 1e8, 0.15, 0.03, 16, 128, 512, 64)
    for nodes, expected in ((2001, 0), (2002, _lib.ERR_UNSUPPORTED)):
        offs = np.zeros(nodes + 1, dtype=np.int32)
        offs[1:] = np.minimum(np.arange(1, nodes + 1), nodes - 1)     # node n's child is n + 1
        kids = np.arange(1, nodes, dtype=np.int32)
        sizes = np.ones(nodes, dtype=np.int32)
        roffs = np.arange(nodes + 1, dtype=np.int32)
        runs = np.stack([np.arange(nodes), np.ones(nodes, dtype=np.int64)], axis=1).astype(np.int64).ravel()
        pushed = np.zeros(nodes, dtype=np.uint8)
        for method in (_lib.SCHEDULE_GREEDY, _lib.SCHEDULE_CUBE):
            rc = lib.ta_schedule_tree(offs.ctypes.data, kids.ctypes.data, sizes.ctypes.data, roffs.ctypes.data,
                                      runs.ctypes.data, nodes, method, ctypes.byref(model), 32, 8, 128,
                                      pushed.ctypes.data, None)
            assert rc == expected, (nodes, method)
