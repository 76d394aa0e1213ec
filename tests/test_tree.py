"""Radix tree vs the reference's own trees (fixtures from tests/golden/make_golden.py)."""
import json
from pathlib import Path

import pytest

from tree_attention import KVTree
from tests.golden.make_golden import TREE_SPECS, build_tree, dump_tree

GOLDEN = json.loads((Path(__file__).parent / "golden" / "trees.json").read_text())


class _Lib:
    KVTree = KVTree


@pytest.mark.parametrize("spec", TREE_SPECS, ids=[s["name"] for s in TREE_SPECS])
def test_tree_matches_reference(spec):
    tree = build_tree(_Lib, spec)
    assert dump_tree(tree) == GOLDEN[spec["name"]]["tree"]


def test_storage_tokens_with_duplicates_and_internal_terminal():
    # reference tests/test_semantics.py:11-13
    tree = KVTree.from_sequences([[1, 2, 3], [1, 2], [1, 2, 4, 5, 6], [7, 8], [1, 2, 3]])
    assert tree.storage_tokens == 8
    assert tree.paths[0] == tree.paths[4]
    assert tree.token_ids == [1, 2, 3, 4, 5, 6, 7, 8]


def test_extension_keeps_private_paths_compressed():
    # reference tests/test_semantics.py:36-42
    tree = KVTree.from_sequences([[1, 2], [1, 2], [3, 4]])
    leaves = [next(i for i, n in enumerate(tree.nodes) if r in n.terminal) for r in range(3)]
    tree.extend_leaves(leaves, [4, 5, 6])
    assert len(tree.nodes) == 5
    tree.extend_leaves(leaves, [7, 8, 9])
    assert len(tree.nodes) == 5


@pytest.mark.parametrize("bad", [[], [[1], []]])
def test_empty_context_rejected(bad):
    with pytest.raises(ValueError):
        KVTree.from_sequences(bad)


def test_synthetic_validation():
    with pytest.raises(ValueError):
        KVTree.synthetic([-1, 2, 0], [1, 1, 1], [1])
    with pytest.raises(ValueError):
        KVTree.synthetic([0], [1], [0])
    with pytest.raises(ValueError):
        KVTree.synthetic([-1, 0], [0, 0], [1])


def test_deep_chain_does_not_recurse():
    # 3000 nested branch points: an iterative builder handles what recursion cannot
    seqs = [[0] * i + [1] for i in range(1, 3000, 1)][:200] + [[0] * 3000]
    tree = KVTree.from_sequences(seqs)
    assert tree.storage_tokens == 3000 + 200
