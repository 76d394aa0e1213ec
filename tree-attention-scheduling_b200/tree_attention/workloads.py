"""Synthetic request trees for the benchmark configurations.

Each generator returns ``KVTree``s built with ``KVTree.synthetic`` (positions in
node order), seeded and deterministic:

* ``small_tree()``      one 1024-token root, 2 children of 256, 8 private 64-token leaves
* ``headline_tree()``   one 8128-token root shared by 128 requests, 128 private 64-token leaves
* ``decode_tree()``     4096-token root, 4 branches of 1024, 32 private 256-token leaves
* ``evaluation_grid(seed)``   81 shapes: requests {16, 64, 256} x depth {1, 2, 4} x shared
  fraction {0.25, 0.75, 0.99} x branching {2, 4, 16}; per-request context 2048-16384 tokens,
  uneven nested prefixes, requests ending at internal nodes, duplicate requests
* ``calibration_grid(seed)``  shapes for fitting the cost model, disjoint from the evaluation
  grid (other request counts, fractions and branchings)

The reference's own 81-tree evaluation grid (``scripts/tree_shapes.py:5-19``: 4/12/24 requests)
is a different, smaller family; the scheduler tests reproduce it exactly from its definition.
"""
from __future__ import annotations

import random
from itertools import product

from .tree import KVTree


def small_tree():
    parents = [-1, 0, 0] + [1] * 4 + [2] * 4
    lengths = [1024, 256, 256] + [64] * 8
    return KVTree.synthetic(parents, lengths, list(range(3, 11)))


def headline_tree(requests=128, root=8128, leaf=64):
    return KVTree.synthetic([-1] + [0] * requests, [root] + [leaf] * requests, list(range(1, requests + 1)))


def decode_tree(root=4096, branches=4, branch_len=1024, requests=32, leaf=256):
    parents = [-1] + [0] * branches + [1 + r * branches // requests for r in range(requests)]
    lengths = [root] + [branch_len] * branches + [leaf] * requests
    return KVTree.synthetic(parents, lengths, list(range(1 + branches, 1 + branches + requests)))


def nested_tree(rng, requests, depth, shared_fraction, branching, context,
                end_inside=0.05, duplicates=0.05):
    """A tree whose shared part has ``depth`` levels of ``branching``-way splits.

    Every request's context is about ``context`` tokens, of which about
    ``shared_fraction`` lie in internal (shared) nodes; level lengths and leaf
    lengths are jittered so prefixes are uneven.  A fraction of the requests
    end at an internal node (no private leaf) and a fraction duplicate another
    request's context exactly.
    """
    shared = max(1, int(round(shared_fraction * context)))
    weights = [rng.uniform(0.6, 1.4) for _ in range(depth)]
    level_len = [max(1, int(shared * w / sum(weights))) for w in weights]
    parents, lengths, level_nodes = [-1], [level_len[0]], [[0]]
    for d in range(1, depth):
        nodes = []
        for parent in level_nodes[-1]:
            for _ in range(branching):
                if len(nodes) >= requests:
                    break
                parents.append(parent)
                lengths.append(max(1, int(level_len[d] * rng.uniform(0.7, 1.3))))
                nodes.append(len(parents) - 1)
        level_nodes.append(nodes)
    deepest = level_nodes[-1]
    terminals = []
    for r in range(requests):
        node = deepest[r % len(deepest)]
        if r > 0 and rng.random() < duplicates:
            terminals.append(terminals[rng.randrange(r)])      # same context as an earlier request
            continue
        if rng.random() < end_inside:
            # ends at an internal node of its branch: no private tokens
            internal = [node]
            while parents[internal[-1]] >= 0:
                internal.append(parents[internal[-1]])
            terminals.append(rng.choice(internal))
            continue
        path_len = 0
        n = node
        while n >= 0:
            path_len += lengths[n]
            n = parents[n]
        parents.append(node)
        lengths.append(max(1, int(max(1, context - path_len) * rng.uniform(0.75, 1.25))))
        terminals.append(len(parents) - 1)
    return KVTree.synthetic(parents, lengths, terminals)


EVALUATION_AXES = dict(requests=(16, 64, 256), depth=(1, 2, 4), shared_fraction=(0.25, 0.75, 0.99),
                       branching=(2, 4, 16))
CONTEXTS = (2048, 4096, 8192, 16384)


def evaluation_grid(seed=201):
    """The 81 evaluation shapes as ``(parameters, tree)`` pairs."""
    for index, (requests, depth, frac, branching) in enumerate(product(*EVALUATION_AXES.values())):
        rng = random.Random(seed * 1000 + index)
        context = CONTEXTS[index % len(CONTEXTS)]
        tree = nested_tree(rng, requests, depth, frac, branching, context)
        params = dict(requests=requests, depth=depth, shared_fraction=frac, branching=branching, context=context)
        yield params, tree


CALIBRATION_AXES = dict(requests=(8, 32, 128), depth=(1, 3), shared_fraction=(0.5, 0.9), branching=(3, 8))


def calibration_grid(seed=501):
    """Shapes for fitting the cost model; no request count, fraction or branching of the evaluation grid."""
    for index, (requests, depth, frac, branching) in enumerate(product(*CALIBRATION_AXES.values())):
        rng = random.Random(seed * 1000 + index)
        context = (1536, 3072, 6144)[index % 3]
        tree = nested_tree(rng, requests, depth, frac, branching, context)
        params = dict(requests=requests, depth=depth, shared_fraction=frac, branching=branching, context=context)
        yield params, tree
