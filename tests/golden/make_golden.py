"""Generate the golden fixtures in this directory from the reference itself.

Run where the reference source is available (it is not on the GPU machines):

    python tests/golden/make_golden.py /path/to/tree-attention-scheduling

It imports the reference's own ``src/tree_attention`` package (tree, schedule,
kernels.prepare on CPU tensors, reference) and records:

* ``trees.json``    node tables, paths and storage order of a set of trees,
                    including trees grown with ``extend_leaves``;
* ``plans.json``    job lists and estimated costs (as float.hex) of every
                    method x cost model x head configuration on those trees,
                    the 81-tree scan of ``scripts/scan_trees.py`` and the
                    reference's 81-tree evaluation grid (``scripts/tree_shapes.py``);
* ``headline_plan.json`` the reference's cube plan of the headline tree with
                    its default cost model, job by job (the reference arm of
                    ``bench.py`` times the oracle on it);
* ``prepare.npz``   the int32 metadata arrays of ``kernels.prepare``;
* ``attention.npz`` seeded inputs with the FP32 outputs of
                    ``reference.request_attention`` / ``segmented_attention``.

The fixtures are committed; tests read them without the reference.
"""
from __future__ import annotations

import hashlib
import importlib
import itertools
import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent

# Trees are described as data so the product tests can rebuild them.
TREE_SPECS = [
    {"name": "unequal_nested_terminal", "sequences": [[1, 2, 3], [1, 2], [1, 2, 4, 5, 6], [7, 8], [1, 2, 3]]},
    {"name": "no_shared_prefix", "sequences": [[1, 2, 3], [4], [5, 6, 7, 8, 9]]},
    {"name": "deep_synthetic", "synthetic": [[-1, 0, 1, 1, 0], [129, 65, 17, 33, 81], [2, 3, 4]]},
    {"name": "duplicate_terminal", "sequences": [[1, 2], [1, 2], [1, 2, 3, 4], [1, 5, 6]]},
    {"name": "wide", "synthetic": [[-1] + [0] * 32, [257] + [31 + i for i in range(32)], list(range(1, 33))]},
    {"name": "extension", "sequences": [[1, 2], [1, 2], [3, 4]], "extend": [[4, 5, 6], [7, 8, 9]]},
    {"name": "small_config1", "synthetic": [[-1, 0, 0] + [1] * 4 + [2] * 4, [1024, 256, 256] + [64] * 8,
                                            list(range(3, 11))]},
    {"name": "mini_config1", "synthetic": [[-1, 0, 0] + [1] * 4 + [2] * 4, [96, 32, 32] + [8] * 8,
                                           list(range(3, 11))]},
    {"name": "headline", "synthetic": [[-1] + [0] * 128, [8128] + [64] * 128, list(range(1, 129))]},
    {"name": "decode_tree", "synthetic": [[-1, 0, 0, 0, 0] + [1 + i // 8 for i in range(32)],
                                          [4096, 1024, 1024, 1024, 1024] + [256] * 32, list(range(5, 37))]},
    {"name": "deep_bench", "synthetic": [[-1, 0, 1, 1, 2, 2, 3, 3] + list(range(4, 8)) * 4,
                                         [512] * 8 + [64] * 16, list(range(8, 24))]},
    {"name": "no_share_root0", "synthetic": [[-1] + [0] * 8, [0] + [300] * 8, list(range(1, 9))]},
]

COST_MODELS = [
    {},
    {"kv_split": 48},
    {"kv_split": 128},
    {"max_query_rows": 16, "kv_split": 100},
    {"cube_rows": 4, "key_tile": 64},
    {"bandwidth": 6_000_000.0, "cube_flops": 1_200_000_000.0, "task_us": 0.02, "merge_us": 0.002,
     "key_tile": 256, "kv_split": 2048, "max_query_rows": 512},
]
HEADS = [(32, 8, 128), (8, 2, 32)]
METHODS = ("request", "fixed", "greedy", "cube")


def runs(tokens):
    out = []
    for p in tokens:
        if out and p == out[-1][0] + out[-1][1]:
            out[-1][1] += 1
        else:
            out.append([p, 1])
    return out


def build_tree(ref, spec):
    if "sequences" in spec:
        tree = ref.KVTree.from_sequences(spec["sequences"])
    else:
        tree = ref.KVTree.synthetic(*spec["synthetic"])
    if "extend" in spec:
        leaves = [next(i for i, n in enumerate(tree.nodes) if r in n.terminal) for r in range(len(tree.paths))]
        for step in spec["extend"]:
            tree.extend_leaves(leaves, step)
    return tree


def dump_tree(tree):
    return {"nodes": [[n.parent, runs(n.tokens), list(n.children), list(n.terminal), list(n.requests)]
                      for n in tree.nodes],
            "paths": [runs(p) for p in tree.paths], "token_ids": tree.token_ids,
            "storage_tokens": tree.storage_tokens}


def plan_digest(jobs):
    """sha256 of the canonical job list: [[requests], [[start, length], ...]] per job."""
    canon = json.dumps([[list(j.requests), runs(j.tokens)] for j in jobs], separators=(",", ":"))
    return hashlib.sha256(canon.encode()).hexdigest()


def dump_plan(plan, full=False):
    row = {"digest": plan_digest(plan.jobs), "njobs": len(plan.jobs), "method": plan.method,
           "estimated_us": float(plan.estimated_us).hex(), "settings": plan.settings}
    if full:
        row["jobs"] = [[list(j.requests), runs(j.tokens)] for j in plan.jobs]
    return row


def reference_grid_trees(ref):
    # scripts/tree_shapes.py:5-19 of the reference: the 81-tree evaluation grid.
    for fanout, root, shared, private in itertools.product(((3, 1), (9, 3), (17, 7)), (32, 192, 768),
                                                          (12, 96, 384), (24, 192, 768)):
        parents, lengths, terminals = [-1], [root], []
        for branch, width in enumerate(fanout):
            node = len(parents)
            parents.append(0)
            lengths.append(shared * (branch + 1) + 7 * branch)
            for leaf in range(width):
                terminals.append(len(parents))
                parents.append(node)
                lengths.append(private * (1 + leaf % 3) + 5 * branch)
        yield [parents, lengths, terminals]


def headline_plan(ref, sched):
    """The reference's own subset-DP plan of the headline tree with its default CostModel(), in full.

    ``bench.py --impl reference`` times the FP32 oracle on this job list, so the reference arm plans
    with the reference's scheduler and cost model and needs nothing from this repository's package.
    """
    spec = next(s for s in TREE_SPECS if s["name"] == "headline")
    tree = build_tree(ref, spec)
    plan = sched.schedule(tree, 32, 8, 128, "cube", sched.CostModel())
    row = dump_plan(plan, full=True)
    row.update(tree=spec["synthetic"], heads=[32, 8, 128], cost_model="CostModel() (reference defaults)")
    return row


def main(reference_root, only_headline=False):
    sys.path.insert(0, str(Path(reference_root) / "src"))
    ref = importlib.import_module("tree_attention")
    sched = importlib.import_module("tree_attention.schedule")
    kernels = importlib.import_module("tree_attention.kernels")
    oracle = importlib.import_module("tree_attention.reference")
    (HERE / "headline_plan.json").write_text(json.dumps(headline_plan(ref, sched)))
    if only_headline:
        return

    trees, plans, prep = {}, [], {}
    for spec in TREE_SPECS:
        tree = build_tree(ref, spec)
        trees[spec["name"]] = {"spec": spec, "tree": dump_tree(tree)}
        for mi, model in enumerate(COST_MODELS):
            for qh, kh, d in HEADS:
                if spec["name"] == "headline" and (qh, kh) != (32, 8):
                    continue
                for method in METHODS:
                    plan = sched.schedule(tree, qh, kh, d, method, sched.CostModel(**model))
                    small = spec["name"] in ("unequal_nested_terminal", "no_shared_prefix", "extension",
                                             "duplicate_terminal")
                    plans.append({"tree": spec["name"], "model": mi, "heads": [qh, kh, d], "method": method,
                                  "plan": dump_plan(plan, full=small and mi == 0)})
                    if mi in (0, 5) and (qh, kh) == (32, 8) or (spec["name"] in ("deep_synthetic",
                                                                                    "unequal_nested_terminal")
                                                               and mi == 1):
                        q = torch.empty(len(tree.paths), qh, d)
                        p = kernels.prepare(plan, q)
                        key = f"{spec['name']}|{mi}|{qh}|{method}"
                        prep[key + "|order"] = np.array(
                            [x for j in p.jobs for x in (len(j.requests), j.tokens[0], len(j.tokens))] +
                            [r for j in p.jobs for r in j.requests], dtype=np.int64)
                        for name in ("qids", "kids", "qlen", "klen", "slots", "counts"):
                            prep[f"{key}|{name}"] = getattr(p, name).numpy().copy()
                        prep[key + "|flags"] = np.array([p.small_jobs, p.contiguous_k, p.contiguous_q],
                                                        dtype=np.int64)

    scan = []
    for root, child, left, right in itertools.product((16, 128, 1024), (8, 64, 256), (16, 128, 512),
                                                      (16, 128, 512)):
        lengths = [root, child, child, left, right, left, right]
        tree = ref.KVTree.synthetic([-1, 0, 0, 1, 1, 2, 2], lengths, [3, 4, 5, 6])
        row = {"lengths": lengths}
        for method in METHODS:
            plan = sched.schedule(tree, method=method)
            row[method] = [float(plan.estimated_us).hex(), len(plan.jobs)]
        scan.append(row)
    grid = []
    for tree_args in reference_grid_trees(ref):
        tree = ref.KVTree.synthetic(*tree_args)
        row = {"synthetic": tree_args}
        for method in METHODS:
            plan = sched.schedule(tree, method=method)
            row[method] = dump_plan(plan)
        grid.append(row)

    attention = {}
    cases = [("unequal_nested_terminal", 8, 2, 32, 1.0, 17), ("no_shared_prefix", 8, 2, 32, 1.0, 17),
             ("deep_synthetic", 8, 2, 32, 30.0, 17), ("extension", 8, 2, 32, 1.0, 17),
             ("duplicate_terminal", 8, 2, 64, 1.0, 2026), ("mini_config1", 32, 8, 128, 1.0, 101)]
    for name, qh, kh, d, scale, seed in cases:
        tree = build_tree(ref, trees[name]["spec"])
        torch.manual_seed(seed)
        # bf16-representable inputs (stored as their bf16 bit patterns) keep
        # the fixture small; the reference computes on their float32 values.
        q = (torch.randn(len(tree.paths), qh, d) * scale).bfloat16()
        k = torch.randn(tree.storage_tokens, kh, d).bfloat16()
        v = torch.randn_like(k, dtype=torch.float32).bfloat16()
        key = f"{name}|{qh}|{kh}|{d}|{scale}"
        for tag, t in (("q", q), ("k", k), ("v", v)):
            attention[f"{key}|{tag}"] = t.view(torch.int16).numpy().view(np.uint16)
        q, k, v = q.float(), k.float(), v.float()
        attention[key + "|request"] = oracle.request_attention(q, k, v, tree).numpy()
        model = sched.CostModel(kv_split=48) if d == 32 else sched.CostModel()
        for method in METHODS:
            plan = sched.schedule(tree, qh, kh, d, method, model)
            attention[f"{key}|{method}"] = oracle.segmented_attention(q, k, v, plan).numpy()

    (HERE / "trees.json").write_text(json.dumps(trees))
    (HERE / "plans.json").write_text(json.dumps({"cost_models": COST_MODELS, "plans": plans, "scan": scan,
                                                  "reference_grid": grid}))
    np.savez_compressed(HERE / "prepare.npz", **prep)
    np.savez_compressed(HERE / "attention.npz", **attention)
    print("trees", len(trees), "plans", len(plans), "prepare", len(prep), "attention", len(attention))


if __name__ == "__main__":
    args = [a for a in sys.argv[1:] if a != "--headline-plan-only"]
    if len(args) != 1:
        sys.exit("usage: python tests/golden/make_golden.py [--headline-plan-only] /path/to/tree-attention-scheduling")
    main(args[0], only_headline="--headline-plan-only" in sys.argv)
