"""KV-head sharding over several ranks, on CPU with the gloo backend (world size 2).

The decode path shards by KV head: rank r owns KV heads [r*HK/N, (r+1)*HK/N),
their query heads and that slice of the pools; the plan is head-independent and
identical on every rank; attention needs no collective, and the Qwen adapter
all-gathers the attention output of each layer before o_proj.  These tests run
that host logic in two gloo processes, with the FP32 oracle standing in for the
CUDA kernels, and compare against the unsharded result.
"""
import os
import socket
import sys
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    sys.path.insert(0, str(ROOT / "tree-attention-scheduling_b200"))
    sys.path.insert(0, str(ROOT))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))


def _attention_worker(rank, world, port, results):
    _init(rank, world, port)
    try:
        from oracle import attention as oracle
        from tree_attention import CostModel, KVTree, kernels, schedule
        hq, hk, d = 32, 8, 128
        tree = KVTree.synthetic([-1, 0, 0, 1, 1, 2], [300, 40, 90, 17, 5, 60], [3, 4, 5, 3, 2, 4])
        nreq = len(tree.paths)
        g = torch.Generator().manual_seed(7)
        q = torch.randn(nreq, hq, d, generator=g)
        k = torch.randn(tree.storage_tokens, hk, d, generator=g)
        v = torch.randn(tree.storage_tokens, hk, d, generator=g)
        plan = schedule(tree, hq, hk, d, "cube", CostModel.b200())
        local_hk, local_hq = hk // world, hq // world
        heads = slice(rank * local_hk, (rank + 1) * local_hk)
        qheads = slice(rank * local_hq, (rank + 1) * local_hq)
        q_local = q[:, qheads].contiguous().bfloat16()
        prepared = kernels.prepare(plan, q_local, num_kv_heads=local_hk)
        # the plan metadata is identical on every rank
        import hashlib
        sha = hashlib.sha256(prepared.metadata.numpy().tobytes()).digest()
        digest = torch.tensor([int.from_bytes(sha[:7], "little")], dtype=torch.int64)
        digests = [torch.zeros_like(digest) for _ in range(world)]
        dist.all_gather(digests, digest)
        same = all(int(x) == int(digest) for x in digests)
        # each rank's shard of the attention, then an all-gather along the heads
        local = oracle.segmented_attention(q[:, qheads], k[:, heads], v[:, heads], plan.jobs)
        gathered = torch.empty((world * nreq, local_hq, d))
        dist.all_gather_into_tensor(gathered, local.contiguous())
        out = gathered.view(world, nreq, local_hq, d).permute(1, 0, 2, 3).reshape(nreq, hq, d)
        full = oracle.segmented_attention(q, k, v, plan.jobs)
        results[rank] = (same, float((out - full).abs().max()))
    finally:
        dist.destroy_process_group()


def _qwen_worker(rank, world, port, results):
    _init(rank, world, port)
    try:
        sys.path.insert(0, str(ROOT / "tests"))
        import test_qwen as tq
        from tree_attention import qwen
        model = tq.tiny_model(32, 4, 2, torch.float32, "cpu")
        decoder = qwen.SharedKVDecoder(model, [list(s) for s in tq.SEQUENCES], max_new_tokens=3, method="cube",
                                       shard=(rank, world, None))
        qwen.attention_matrix = tq.oracle_attention(decoder)
        qwen.append_kv = tq.reference_append
        logits = [decoder.logits.clone()]
        for _ in range(2):
            tokens = decoder.logits.argmax(-1).tolist()
            logits.append(decoder.step(tokens).clone())
        reference = tq.reference_logits(model, decoder.sequences)
        results[rank] = (float((logits[-1] - reference).abs().max()), decoder.pools[0][0].shape[0])
    finally:
        dist.destroy_process_group()


def _max_worker(rank, world, port, results):
    _init(rank, world, port)
    try:
        import bench
        results[rank] = bench.max_over_ranks(10.0 + rank, world)
    finally:
        dist.destroy_process_group()


def _run(worker, world=2):
    manager = mp.get_context("spawn").Manager()
    results = manager.dict()
    mp.start_processes(worker, args=(world, _free_port(), results), nprocs=world, start_method="spawn", join=True)
    return dict(results)


def test_kv_head_shards_reassemble_the_full_attention():
    results = _run(_attention_worker)
    assert len(results) == 2
    for same, err in results.values():
        assert same
        assert err < 1e-5


def test_qwen_decoder_sharded_over_two_ranks():
    pytest.importorskip("transformers")
    results = _run(_qwen_worker)
    assert len(results) == 2
    for err, local_heads in results.values():
        assert local_heads == 1                 # 2 KV heads over 2 ranks
        assert err < 1e-4


def test_step_time_is_the_max_over_ranks():
    results = _run(_max_worker)
    assert results == {0: 11.0, 1: 11.0}
