"""The CPU oracle against golden outputs of the reference's own reference.py."""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import attention as oracle
from tree_attention import CostModel, KVTree, schedule
from tests.golden.make_golden import TREE_SPECS, build_tree

ATT = np.load(Path(__file__).parent / "golden" / "attention.npz")
SPECS = {s["name"]: s for s in TREE_SPECS}
CASES = sorted({k.rsplit("|", 1)[0] for k in ATT.files})


class _Lib:
    KVTree = KVTree


def load_bf16(key):
    return torch.from_numpy(ATT[key].view(np.int16).copy()).view(torch.bfloat16).float()


@pytest.mark.parametrize("case", CASES)
def test_oracle_matches_reference(case):
    name, qh, kh, d, scale = case.split("|")
    qh, kh, d = int(qh), int(kh), int(d)
    tree = build_tree(_Lib, SPECS[name])
    q, k, v = (load_bf16(f"{case}|{t}") for t in "qkv")
    expected = torch.from_numpy(ATT[f"{case}|request"])
    out = oracle.request_attention(q, k, v, tree.paths)
    torch.testing.assert_close(out, expected, atol=2e-6, rtol=2e-6)
    model = CostModel(kv_split=48) if d == 32 else CostModel()
    for method in ("request", "fixed", "greedy", "cube"):
        plan = schedule(tree, qh, kh, d, method, model)
        seg = oracle.segmented_attention(q, k, v, plan.jobs)
        torch.testing.assert_close(seg, torch.from_numpy(ATT[f"{case}|{method}"]), atol=2e-6, rtol=2e-6)
        # and the oracle's two formulations agree (reference tests/test_semantics.py:34)
        torch.testing.assert_close(seg, out, atol=2e-5, rtol=2e-5)


def test_lse_matches_logsumexp():
    torch.manual_seed(0)
    tree = KVTree.synthetic([-1, 0, 0], [40, 7, 9], [1, 2, 2])
    q = torch.randn(3, 8, 32)
    k = torch.randn(tree.storage_tokens, 2, 32)
    v = torch.randn_like(k)
    _, out_f, lse = oracle.request_attention(q, k, v, tree.paths, return_lse=True)
    plan = schedule(tree, 8, 2, 32, "cube", CostModel(kv_split=16))
    _, seg_f, seg_lse = oracle.segmented_attention(q, k, v, plan.jobs, return_lse=True)
    torch.testing.assert_close(seg_f, out_f, atol=2e-5, rtol=2e-5)
    torch.testing.assert_close(seg_lse, lse, atol=2e-5, rtol=2e-5)
    r = 1
    s = torch.einsum("hd,nhd->hn", q[r], k[list(tree.paths[r])].repeat_interleave(4, 1)) / 32 ** 0.5
    torch.testing.assert_close(lse[r], torch.logsumexp(s, -1))


def test_oracle_detects_planted_error():
    """A mistake planted in the oracle's input plan is caught by the comparison."""
    tree = KVTree.synthetic([-1, 0, 0], [40, 7, 9], [1, 2])
    torch.manual_seed(1)
    q = torch.randn(2, 8, 32)
    k = torch.randn(tree.storage_tokens, 2, 32)
    v = torch.randn_like(k)
    plan = schedule(tree, 8, 2, 32, "fixed", CostModel())
    from tree_attention.schedule import Job
    broken = [Job(j.requests, j.tokens[:-1]) if len(j.tokens) > 1 else j for j in plan.jobs]
    good = oracle.request_attention(q, k, v, tree.paths)
    bad = oracle.segmented_attention(q, k, v, broken)
    assert not torch.allclose(good, bad, atol=1e-3)


def test_oracle_takes_the_reference_arguments():
    """The reference's scripts call reference.request_attention(q, k, v, tree) and
    segmented_attention(q, k, v, plan): the oracle accepts those objects too."""
    case = CASES[0]
    name, qh, kh, d, _ = case.split("|")
    tree = build_tree(_Lib, SPECS[name])
    q, k, v = (load_bf16(f"{case}|{t}") for t in "qkv")
    plan = schedule(tree, int(qh), int(kh), int(d), "cube", CostModel(kv_split=48) if int(d) == 32 else CostModel())
    assert torch.equal(oracle.request_attention(q, k, v, tree), oracle.request_attention(q, k, v, tree.paths))
    assert torch.equal(oracle.segmented_attention(q, k, v, plan), oracle.segmented_attention(q, k, v, plan.jobs))
