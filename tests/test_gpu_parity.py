"""Kernel parity on a B200: the CUDA path through the C ABI against the FP32 oracle.

Tolerances (north-star criteria): per-(request, head) relative L2 <= 5e-3 of
the BF16 output against the FP32 oracle, |dLSE| <= 1e-3 in natural-log units;
plus the reference's own benchmark check atol .008 / rtol .03
(scripts/benchmark.py:96 of the reference).
"""
import os

import pytest
import torch

from oracle import attention as oracle
from tree_attention import CostModel, KVTree, schedule
from tree_attention import kernels
from tree_attention.kernels import CachedDecodePlan, attention_matrix, check_status, pack_kv, prepare
from tests.golden.make_golden import TREE_SPECS, build_tree

pytestmark = pytest.mark.gpu

REL_L2 = 5e-3
LSE_TOL = 1e-3
SPECS = {s["name"]: s for s in TREE_SPECS}


class _Lib:
    KVTree = KVTree


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    os.environ["TREE_ATTN_CHECK"] = "1"
    yield
    os.environ.pop("TREE_ATTN_CHECK", None)


def make_inputs(nreq, storage, hq, hk, d, dtype, seed, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    q = (torch.randn(nreq, hq, d, generator=g) * scale).to(dtype)
    k = torch.randn(storage, hk, d, generator=g).to(dtype)
    v = torch.randn(storage, hk, d, generator=g).to(dtype)
    return q, k, v


def rel_l2(actual, expected):
    err = (actual.float() - expected.float()).flatten(2).norm(dim=-1)
    ref = expected.float().flatten(2).norm(dim=-1).clamp_min(1e-30)
    return (err / ref)


def run_kernel(q, k, v, plan, pool_pad=0, pad_value=float("nan")):
    dev = "cuda"
    qd = q.to(dev)
    kp, vp = pack_kv(k.to(dev), v.to(dev))
    if pool_pad:
        # capacity beyond the used positions holds garbage (NaN) that must never be read
        pad = torch.full((kp.shape[0], pool_pad, kp.shape[2]), pad_value, dtype=kp.dtype, device=dev)
        kp = torch.cat([kp, pad], 1).contiguous()
        vp = torch.cat([vp, pad], 1).contiguous()
    p = prepare(plan, qd)
    lse = torch.empty(q.shape[0], q.shape[1], device=dev, dtype=torch.float32)
    out = attention_matrix(qd, kp, vp, p, out_lse=lse)
    torch.cuda.synchronize()
    check_status(p)
    return out.cpu(), lse.cpu(), p


def check_against_oracle(q, k, v, paths, out, lse):
    _, ref_f, ref_lse = oracle.request_attention(q.float(), k.float(), v.float(), paths, return_lse=True)
    err = rel_l2(out, ref_f)
    assert torch.isfinite(out.float()).all()
    assert err.max().item() <= REL_L2, f"max rel L2 {err.max().item():.3e}"
    assert (lse - ref_lse).abs().max().item() <= LSE_TOL
    torch.testing.assert_close(out.float(), ref_f.to(out.dtype).float(), atol=.008, rtol=.03)


TREES = ["unequal_nested_terminal", "no_shared_prefix", "deep_synthetic", "duplicate_terminal", "wide",
         "extension", "small_config1", "deep_bench", "no_share_root0", "decode_tree"]


@pytest.mark.parametrize("name", TREES)
@pytest.mark.parametrize("heads", [(32, 8, 128), (8, 2, 64), (8, 2, 32)], ids=["h32x8d128", "h8x2d64", "h8x2d32"])
def test_tree_plans_match_oracle(name, heads):
    hq, hk, d = heads
    tree = build_tree(_Lib, SPECS[name])
    q, k, v = make_inputs(len(tree.paths), tree.storage_tokens, hq, hk, d, torch.bfloat16, seed=101)
    for model in (CostModel(), CostModel(kv_split=48), CostModel.b200()):
        for method in ("request", "fixed", "greedy", "cube"):
            plan = schedule(tree, hq, hk, d, method, model)
            out, lse, _ = run_kernel(q, k, v, plan, pool_pad=37)
            check_against_oracle(q, k, v, tree.paths, out, lse)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_reference_check_trees(dtype):
    """The reference's scripts/check_npu.py:12-31 trees, both dtypes, kv_split=128."""
    trees = {
        "unequal": KVTree.synthetic([-1, 0, 0, 1, 1], [129, 65, 17, 33, 81], [2, 3, 4]),
        "none": KVTree.from_sequences([[1, 2, 3], [4], [5, 6, 7, 8, 9]]),
        "duplicate_terminal": KVTree.from_sequences([[1, 2], [1, 2], [1, 2, 3, 4], [1, 5, 6]]),
        "wide": KVTree.synthetic([-1] + [0] * 32, [257] + [31 + i for i in range(32)], list(range(1, 33))),
    }
    for tree in trees.values():
        q, k, v = make_inputs(len(tree.paths), tree.storage_tokens, 8, 2, 64, dtype, seed=2026)
        for method in ("request", "fixed", "greedy", "cube"):
            plan = schedule(tree, 8, 2, 64, method, CostModel(kv_split=128))
            out, lse, _ = run_kernel(q, k, v, plan)
            check_against_oracle(q, k, v, tree.paths, out, lse)


def test_extreme_logits():
    """Scores scaled x30 stress the LSE merge (reference tests/test_semantics.py:19-21)."""
    tree = build_tree(_Lib, SPECS["deep_synthetic"])
    q, k, v = make_inputs(len(tree.paths), tree.storage_tokens, 8, 2, 32, torch.bfloat16, seed=17, scale=30.0)
    for method in ("request", "fixed", "greedy", "cube"):
        plan = schedule(tree, 8, 2, 32, method, CostModel(kv_split=48))
        out, lse, _ = run_kernel(q, k, v, plan)
        check_against_oracle(q, k, v, tree.paths, out, lse)


def test_segment_partials_match_oracle():
    """Each (piece, request) partial output and LSE, read back from the scratch buffers."""
    tree = build_tree(_Lib, SPECS["deep_bench"])
    q, k, v = make_inputs(len(tree.paths), tree.storage_tokens, 32, 8, 128, torch.bfloat16, seed=5)
    plan = schedule(tree, 32, 8, 128, "cube", CostModel(kv_split=200))
    _, _, p = run_kernel(q, k, v, plan)
    part, lse = p.part.cpu(), p.lse.cpu()
    pieces = p.host_arrays["pieces"]
    piece_jobs = [kernels.Job(p.jobs[j].requests, p.jobs[j].tokens[o:o + n]) for j, o, n, _ in pieces]
    expected = oracle.job_partials(q.float(), k.float(), v.float(), piece_jobs)
    for (_, _, _, first), job, (o_ref, l_ref) in zip(pieces, piece_jobs, expected):
        for j in range(len(job.requests)):
            rows = slice((first + j) * 4, (first + j + 1) * 4)
            o = part[:, rows].reshape(32, 128)      # [HK*G, D] == query heads in order
            l = lse[:, rows].reshape(32)
            assert ((o - o_ref[j]).norm(dim=-1) / o_ref[j].norm(dim=-1)).max() <= REL_L2
            assert (l - l_ref[j]).abs().max() <= LSE_TOL


def test_one_kv_head_many_partials():
    """One KV head (the 8-GPU shard of the headline shape): the root is cut into many pieces, so each
    request merges more partials than one warp's batch and the split merge kernel runs."""
    tree = KVTree.synthetic([-1] + [0] * 64, [8128] + [32] * 64, list(range(1, 65)))
    q, k, v = make_inputs(64, tree.storage_tokens, 4, 1, 128, torch.bfloat16, seed=11)
    plan = schedule(tree, 4, 1, 128, "cube", CostModel.b200())
    out, lse, p = run_kernel(q, k, v, plan, pool_pad=64)
    assert p.layout.max_pslots > 24
    check_against_oracle(q, k, v, tree.paths, out, lse)


def test_large_group_rows():
    """256 requests sharing one prefix: a job of 1024 query rows (many row tiles)."""
    tree = KVTree.synthetic([-1] + [0] * 256, [700] + [3 + (i % 5) for i in range(256)], list(range(1, 257)))
    q, k, v = make_inputs(256, tree.storage_tokens, 32, 8, 128, torch.bfloat16, seed=9)
    plan = schedule(tree, 32, 8, 128, "cube", CostModel.b200())
    out, lse, _ = run_kernel(q, k, v, plan, pool_pad=300)
    check_against_oracle(q, k, v, tree.paths, out, lse)


def test_cached_decode_plan_matches_oracle():
    """Prompt plan reused over decode steps with growing private tails (incl. length 0)."""
    base = KVTree.synthetic([-1, 0, 0, 0, 0] + [1 + i // 2 for i in range(8)], [300, 100, 90, 80, 70] + [40] * 8,
                            list(range(5, 13)))
    steps = 5
    prefix = base.storage_tokens
    q, k, v = make_inputs(8, prefix + 8 * steps, 32, 8, 128, torch.bfloat16, seed=301)
    qd = q.cuda()
    kp, vp = pack_kv(k.cuda(), v.cuda())
    cached = CachedDecodePlan(schedule(base, method="cube", model=CostModel(kv_split=128)), qd, prefix, steps)
    assert cached.tail_indices.numel() == 8
    for n in (0, 1, 3, steps):
        p = cached.update(n)
        lse = torch.empty(8, 32, device="cuda")
        out = attention_matrix(qd, kp, vp, p, out_lse=lse).cpu()
        torch.cuda.synchronize()
        check_status(p)
        paths = [path + tuple(prefix + r * steps + t for t in range(n)) for r, path in enumerate(base.paths)]
        check_against_oracle(q, k, v, paths, out, lse.cpu())


def test_cached_decode_plan_with_long_runs_of_empty_tails():
    """1200 requests with private leaves and a cached decode plan: before the first token every tail is
    empty, and some keys-in-lanes CTAs run 8 or more tasks without tiles in a row after a task with tiles
    (the task ring is 8 slots deep).  The step completes with status OK and matches the oracle, then again
    with one token per tail."""
    nreq, steps = 1200, 2
    base = KVTree.synthetic([-1] + [0] * nreq, [512] + [16] * nreq, list(range(1, nreq + 1)))
    prefix = base.storage_tokens
    q, k, v = make_inputs(nreq, prefix + nreq * steps, 32, 8, 128, torch.bfloat16, seed=303)
    qd = q.cuda()
    kp, vp = pack_kv(k.cuda(), v.cuda())
    cached = CachedDecodePlan(schedule(base, 32, 8, 128, "cube", CostModel.b200()), qd, prefix, steps)
    sample = list(range(0, nreq, 97)) + [nreq - 1]
    for n in (0, 1):
        p = cached.update(n)
        lse = torch.empty(nreq, 32, device="cuda")
        out = attention_matrix(qd, kp, vp, p, out_lse=lse).cpu()
        torch.cuda.synchronize()
        check_status(p)
        paths = [base.paths[r] + tuple(prefix + r * steps + t for t in range(n)) for r in sample]
        check_against_oracle(q[sample], k, v, paths, out[sample], lse.cpu()[sample])


def test_graph_capture_replays_same_result():
    tree = build_tree(_Lib, SPECS["small_config1"])
    q, k, v = make_inputs(8, tree.storage_tokens, 32, 8, 128, torch.bfloat16, seed=3)
    qd = q.cuda()
    kp, vp = pack_kv(k.cuda(), v.cuda())
    p = prepare(schedule(tree, method="cube", model=CostModel.b200()), qd)
    eager = attention_matrix(qd, kp, vp, p).clone()
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    os.environ["TREE_ATTN_CHECK"] = "0"
    try:
        with torch.cuda.graph(graph, stream=stream):
            attention_matrix(qd, kp, vp, p)
    finally:
        os.environ["TREE_ATTN_CHECK"] = "1"
    p.out.zero_()
    graph.replay()
    torch.cuda.synchronize()
    check_status(p)
    assert torch.equal(p.out, eager)


def test_bounds_violation_is_reported_not_trapped():
    """A pool shorter than the plan's positions: the kernel skips the read and flags it.

    The real allocation is larger than the claimed pool length, so even an
    unchecked access would stay inside memory this process owns.
    """
    tree = KVTree.synthetic([-1, 0, 0], [64, 16, 16], [1, 2])
    q, k, v = make_inputs(2, tree.storage_tokens, 32, 8, 128, torch.bfloat16, seed=4)
    qd = q.cuda()
    kp, vp = pack_kv(k.cuda(), v.cuda())
    p = prepare(schedule(tree, method="fixed"), qd)
    lib = kernels._lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.ta_attention(p.layout, p.metadata.data_ptr(), qd.data_ptr(), kp.data_ptr(), vp.data_ptr(), 70,
                          32, 8, 128, kernels._lib.DTYPE_BF16, p.part.data_ptr(), p.lse.data_ptr(),
                          p.out.data_ptr(), None, p.status.data_ptr(), stream)
    assert rc == 0
    torch.cuda.synchronize()
    assert int(p.status.item()) & kernels._lib.ERR_BOUNDS
    assert torch.isfinite(p.out.float()).all()
    p.status.zero_()


def test_headline_full_size_properties():
    """Full BASELINE headline shape: tree plans agree with the per-request plan, and all 128
    requests of every plan agree with the FP32 oracle."""
    tree = KVTree.synthetic([-1] + [0] * 128, [8128] + [64] * 128, list(range(1, 129)))
    q, k, v = make_inputs(128, tree.storage_tokens, 32, 8, 128, torch.bfloat16, seed=101)
    qd = q.cuda()
    kp, vp = pack_kv(k.cuda(), v.cuda())
    outs = {}
    for method, model in (("request", CostModel()), ("fixed", CostModel()), ("cube", CostModel()),
                          ("cube", CostModel.b200()), ("greedy", CostModel.b200())):
        p = prepare(schedule(tree, method=method, model=model), qd)
        lse = torch.empty(128, 32, device="cuda")
        outs[(method, model.kv_split)] = (attention_matrix(qd, kp, vp, p, out_lse=lse).clone(), lse)
        torch.cuda.synchronize()
        check_status(p)
    base_out, base_lse = outs[("request", 512)]
    for key, (o, l) in outs.items():
        assert rel_l2(o.cpu(), base_out.cpu()).max() <= REL_L2, key
        assert (l - base_lse).abs().max().item() <= LSE_TOL, key
    # every request of every plan against the FP32 oracle (the oracle runs the 128 x 8192 shape in
    # seconds on the host)
    _, ref_f, ref_lse = oracle.request_attention(q.float(), k.float(), v.float(), tree.paths, return_lse=True)
    for key, (o, l) in outs.items():
        assert rel_l2(o.cpu(), ref_f).max() <= REL_L2, key
        assert (l.cpu() - ref_lse).abs().max() <= LSE_TOL, key
        torch.testing.assert_close(o.cpu().float(), ref_f.to(o.dtype).float(), atol=.008, rtol=.03)


@pytest.mark.parametrize("keys", [1, 100, 128, 129, 256, 384, 512, 640, 1000, 2048, 2600])
@pytest.mark.parametrize("nreq", [5, 32, 40])
def test_tensor_core_pipeline_tile_counts(keys, nreq):
    """One shared segment read by nreq requests (tensor-core path for > 16 rows)
    with 1..21 key tiles: every ring wrap-around and barrier phase of the
    pipeline, full and partial last tiles, NaN in the pool past the segment."""
    tree = KVTree.synthetic([-1], [keys], [0] * nreq)
    q, k, v = make_inputs(nreq, keys, 32, 8, 128, torch.bfloat16, seed=keys * 7 + nreq)
    plan = schedule(tree, 32, 8, 128, "fixed", CostModel(kv_split=4096, max_query_rows=4096))
    out, lse, p = run_kernel(q, k, v, plan, pool_pad=200)
    pieces = p.layout.num_pieces
    if nreq * 4 > kernels.KN_ROWS:
        assert p.layout.num_tc_tasks == pieces * ((nreq * 4 + kernels.TC_ROWS - 1) // kernels.TC_ROWS)
    else:
        assert p.layout.num_kn_tasks > 0 and p.layout.num_tc_tasks == 0
    check_against_oracle(q, k, v, tree.paths, out, lse)


@pytest.mark.parametrize("keys", [1, 15, 16, 17, 31, 32, 33, 100, 127, 128, 129, 300, 1000])
@pytest.mark.parametrize("nreq", [1, 3, 4, 5, 8, 9, 16])
def test_keys_in_lanes_rows_and_tiles(keys, nreq):
    """Keys-in-lanes tcgen05 kernel: jobs of 4..64 query rows (cut into segments of
    at most 16 rows; packed tasks of up to 16 rows), partial
    32-key boxes, V rows zeroed up to the next 16-key step, NaN in the pool past
    the segment, multi-tile pieces."""
    tree = KVTree.synthetic([-1], [keys], [0] * nreq)
    q, k, v = make_inputs(nreq, keys, 32, 8, 128, torch.bfloat16, seed=keys * 13 + nreq)
    plan = schedule(tree, 32, 8, 128, "fixed", CostModel(kv_split=4096, max_query_rows=4096))
    out, lse, p = run_kernel(q, k, v, plan, pool_pad=160)
    if nreq * 4 <= kernels.KN_ROWS:
        assert p.layout.num_kn_tasks > 0 and p.layout.num_tc_tasks == 0 and p.layout.num_small_tasks == 0
        first = kernels.kn_class(min(nreq * 4, kernels.KN_TASK_ROWS))
        assert sum(p.layout.kn_class_ctas[c] for c in range(first, 5)) > 0   # packing may add rows
    else:                                                  # more rows: the query-tile kernel, one partial tile
        assert p.layout.num_tc_tasks > 0 and p.layout.num_kn_tasks == 0
    check_against_oracle(q, k, v, tree.paths, out, lse)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_keys_in_lanes_rising_scores_rescale(dtype):
    """Scores that keep rising along the segment force the stale-maximum rescale of
    the sums and of O^T in TMEM on many tiles; plus x30 random logits."""
    nreq, keys = 6, 1500
    tree = KVTree.synthetic([-1, 0, 0], [keys, 40, 40], [1, 1, 2, 2, 1, 2])
    g = torch.Generator().manual_seed(77)
    q = torch.randn(nreq, 32, 128, generator=g)
    k = torch.randn(tree.storage_tokens, 8, 128, generator=g) * 0.2
    v = torch.randn(tree.storage_tokens, 8, 128, generator=g)
    direction = q.reshape(nreq, 8, 4, 128).mean(dim=(0, 2))          # per KV head
    ramp = torch.linspace(0, 150.0, tree.storage_tokens)[:, None, None]   # ~40 log2 units of score
    k = k + ramp * direction[None] / direction.norm(dim=-1, keepdim=True)[None]
    q, k, v = q.to(dtype), k.to(dtype), v.to(dtype)
    for method in ("fixed", "cube", "request"):
        plan = schedule(tree, 32, 8, 128, method, CostModel(kv_split=4096, max_query_rows=4096))
        out, lse, _ = run_kernel(q, k, v, plan)
        check_against_oracle(q, k, v, tree.paths, out, lse)
    q2, k2, v2 = make_inputs(nreq, tree.storage_tokens, 32, 8, 128, dtype, seed=78, scale=30.0)
    for method in ("fixed", "cube", "request"):
        plan = schedule(tree, 32, 8, 128, method, CostModel(kv_split=256))
        out, lse, _ = run_kernel(q2, k2, v2, plan)
        check_against_oracle(q2, k2, v2, tree.paths, out, lse)


def test_evaluation_grid_sample_matches_oracle():
    """A sample of the 81 evaluation-grid shapes (16 requests: every depth, shared
    fraction and branching factor, uneven prefixes, internal terminations,
    duplicates), tree and per-request plans against the FP32 oracle."""
    from tree_attention import workloads
    for index, (params, tree) in enumerate(workloads.evaluation_grid()):
        if params["requests"] != 16 or params["context"] > 4096 or index % 2:
            continue
        q, k, v = make_inputs(16, tree.storage_tokens, 32, 8, 128, torch.bfloat16, seed=200 + index)
        for method in ("cube", "request"):
            plan = schedule(tree, 32, 8, 128, method, CostModel.b200())
            out, lse, _ = run_kernel(q, k, v, plan, pool_pad=64)
            check_against_oracle(q, k, v, tree.paths, out, lse)


def test_decode_tree_plan_reuse_first_and_last_step():
    """configs[3] shape: the cached plan and the rebuilt plan agree with the oracle
    at the first and last of 16 decode steps."""
    import copy
    from tree_attention import workloads
    steps = 16
    base = workloads.decode_tree()
    prefix = base.storage_tokens
    q, k, v = make_inputs(32, prefix + 32 * steps, 32, 8, 128, torch.bfloat16, seed=301)
    qd = q.cuda()
    kp, vp = pack_kv(k.cuda(), v.cuda())
    cached = CachedDecodePlan(schedule(base, 32, 8, 128, "cube", CostModel.b200()), qd, prefix, steps)
    tree = copy.deepcopy(base)
    leaves = list(range(len(base.nodes) - 32, len(base.nodes)))
    for step in range(steps):
        tree.extend_leaves(leaves, [prefix + r * steps + step for r in range(32)])
        if step not in (0, steps - 1):
            continue
        paths = [path + tuple(prefix + r * steps + t for t in range(step + 1)) for r, path in enumerate(base.paths)]
        assert [tuple(p) for p in tree.paths] == paths
        for p in (cached.update(step + 1), prepare(schedule(tree, 32, 8, 128, "cube", CostModel.b200()), qd)):
            lse = torch.empty(32, 32, device="cuda")
            out = attention_matrix(qd, kp, vp, p, out_lse=lse).cpu()
            torch.cuda.synchronize()
            check_status(p)
            check_against_oracle(q, k, v, paths, out, lse.cpu())


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_decode_append_matches_index_copy(dtype):
    """The fused decode-step append writes the same pool rows as the reference's two index_copy_
    calls, takes strided [NREQ, HK, D] rows, sets the tail lengths from a device count, and flags an
    out-of-range target without writing it."""
    g = torch.Generator(device="cuda").manual_seed(11)
    hk, tokens, dim, nreq = 8, 300, 128, 5
    kp = torch.randn(hk, tokens, dim, generator=g, device="cuda").to(dtype)
    vp = torch.randn_like(kp)
    # rows as the adapter has them: k[:, :, 0, :] of a [NREQ, HK, 1, D] view of a [NREQ, 1, HK, D] tensor
    k4 = torch.randn(nreq, 1, hk, dim, generator=g, device="cuda").to(dtype).transpose(1, 2)
    v4 = torch.randn(nreq, 1, hk, dim, generator=g, device="cuda").to(dtype).transpose(1, 2)
    k_new, v_new = k4[:, :, 0, :], v4[:, :, 0, :]
    targets = torch.tensor([7, 299, 0, 150, 42], device="cuda")
    ref_k, ref_v = kp.clone(), vp.clone()
    ref_k.index_copy_(1, targets, k_new.transpose(0, 1))
    ref_v.index_copy_(1, targets, v_new.transpose(0, 1))
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    kernels.append_kv(kp, vp, k_new, v_new, targets, status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert torch.equal(kp, ref_k) and torch.equal(vp, ref_v)

    # tail lengths of a cached plan from a device count, in the same launch
    tree = KVTree.synthetic([-1, 0, 0], [64, 16, 16], [1, 2])
    q = torch.empty(2, 32, 128, device="cuda", dtype=dtype)
    cached = CachedDecodePlan(schedule(tree, method="cube"), q, tree.storage_tokens, 8)
    count = torch.tensor([4], device="cuda")
    kernels.append_kv(kp, vp, k_new, v_new, targets, None, (cached, count, 1))
    torch.cuda.synchronize()
    tails = cached.tail_indices.long()
    assert cached.prepared.klen[tails].tolist() == [5, 5]
    assert int(cached.prepared.status.item()) == 0

    # an out-of-range target is skipped and flagged; the other rows are written
    bad = torch.tensor([7, tokens, 0, 150, 42], device="cuda")
    kernels.append_kv(kp, vp, torch.zeros_like(k_new), torch.zeros_like(v_new), bad, status)
    torch.cuda.synchronize()
    assert int(status.item()) & kernels._lib.ERR_BOUNDS
    assert kp[:, 7].abs().sum().item() == 0 and torch.equal(kp[:, 299], ref_k[:, 299])


def _segment_then_merge(qd, kp, vp, p, lse_out):
    """ta_segment and ta_merge as two calls (the merge kernel), for comparison with ta_attention."""
    lib = kernels._lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    dt = kernels._DTYPES[qd.dtype]
    hq, hk, d = qd.shape[1], kp.shape[0], qd.shape[2]
    out = torch.empty_like(qd)
    assert lib.ta_segment(p.layout, p.metadata.data_ptr(), qd.data_ptr(), kp.data_ptr(), vp.data_ptr(),
                          kp.shape[1], hq, hk, d, dt, p.part.data_ptr(), p.lse.data_ptr(), p.status.data_ptr(),
                          stream) == 0
    assert lib.ta_merge(p.layout, p.metadata.data_ptr(), p.part.data_ptr(), p.lse.data_ptr(), out.data_ptr(),
                        lse_out.data_ptr(), hq, hk, d, dt, p.status.data_ptr(), stream) == 0
    return out


@pytest.mark.parametrize("heads", [(8, 8), (16, 8), (32, 8), (64, 8)], ids=["G1", "G2", "G4", "G8"])
def test_small_group_kernel_group_sizes(heads):
    """The keys-in-lanes kernel with 1, 2, 4 and 8 query heads per KV head: segments of up to 8 query
    rows (several requests per segment for G = 1 and 2, one request for G = 8), shared small groups and
    private leaves of 1..200 keys; ta_attention and ta_segment + ta_merge give identical results."""
    hq, hk = heads
    leaves = [1, 7, 16, 33, 64, 65, 127, 200]
    parents = [-1, 0, 0] + [1] * 4 + [2] * 4
    lengths = [40, 300, 9] + leaves
    tree = KVTree.synthetic(parents, lengths, [3, 3, 4, 5, 6, 7, 8, 9, 10, 10])
    q, k, v = make_inputs(len(tree.paths), tree.storage_tokens, hq, hk, 128, torch.bfloat16, seed=hq * 7)
    qd = q.cuda()
    kp, vp = pack_kv(k.cuda(), v.cuda())
    for method in ("request", "cube", "fixed"):
        plan = schedule(tree, hq, hk, 128, method, CostModel(kv_split=128))
        p = prepare(plan, qd)
        assert p.layout.num_kn_segs > 0
        lse = torch.empty(len(tree.paths), hq, device="cuda")
        out = attention_matrix(qd, kp, vp, p, out_lse=lse).clone()
        torch.cuda.synchronize()
        check_status(p)
        check_against_oracle(q, k, v, tree.paths, out.cpu(), lse.cpu())
        lse2 = torch.empty_like(lse)
        out2 = _segment_then_merge(qd, kp, vp, p, lse2)
        torch.cuda.synchronize()
        check_status(p)
        assert torch.equal(out2, out) and torch.equal(lse2, lse)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_small_group_kernel_beside_query_tiles(dtype):
    """A shared root on the query-tile kernel and 300 private leaves on the keys-in-lanes kernel, which
    is placed on the SMs the query-tile kernel leaves free; more segments than resident CTAs.  Ten
    back-to-back calls and a graph replay of three give the same result as the first call."""
    nreq = 300
    tree = KVTree.synthetic([-1] + [0] * nreq, [2000] + [17 + (i * 13) % 90 for i in range(nreq)],
                            list(range(1, nreq + 1)))
    q, k, v = make_inputs(nreq, tree.storage_tokens, 32, 8, 128, dtype, seed=41)
    qd = q.cuda()
    kp, vp = pack_kv(k.cuda(), v.cuda())
    p = prepare(schedule(tree, 32, 8, 128, "cube", CostModel.b200()), qd)
    assert p.layout.num_tc_tasks > 0 and p.layout.num_kn_segs > 3 * 148
    lse = torch.empty(nreq, 32, device="cuda")
    first = attention_matrix(qd, kp, vp, p, out_lse=lse).clone()
    torch.cuda.synchronize()
    check_status(p)
    check_against_oracle(q, k, v, tree.paths, first.cpu(), lse.cpu())
    os.environ["TREE_ATTN_CHECK"] = "0"
    try:
        for _ in range(10):
            attention_matrix(qd, kp, vp, p)
        torch.cuda.synchronize()
        assert torch.equal(p.out, first)
        stream = torch.cuda.Stream()
        stream.wait_stream(torch.cuda.current_stream())
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for _ in range(3):
                attention_matrix(qd, kp, vp, p)
        p.out.zero_()
        graph.replay()
        torch.cuda.synchronize()
    finally:
        os.environ["TREE_ATTN_CHECK"] = "1"
    check_status(p)
    assert torch.equal(p.out, first)


def test_bounded_wait_gives_up_and_context_recovers():
    """A bounded device wait that runs out (the SIMT kernel's test hook makes every CTA wait on a barrier
    nothing completes) ends the kernel with TA_ERR_TIMEOUT instead of hanging; the context stays usable and
    the next call on the same plan is correct.  No GPU fault is involved: the wait gives up after about a
    second, the CTA waits for its own copies in flight and exits."""
    tree = build_tree(_Lib, SPECS["small_config1"])
    q, k, v = make_inputs(len(tree.paths), tree.storage_tokens, 8, 2, 64, torch.bfloat16, seed=12)
    qd = q.cuda()
    kp, vp = pack_kv(k.cuda(), v.cuda())
    p = prepare(schedule(tree, 8, 2, 64, "cube", CostModel(kv_split=128)), qd)
    assert p.layout.num_small_tasks > 0 and p.layout.num_tc_tasks == 0 and p.layout.num_kn_tasks == 0
    os.environ["TREE_ATTN_CHECK"] = "0"
    os.environ["TREE_ATTN_TEST_STALL"] = "1"
    try:
        attention_matrix(qd, kp, vp, p)
        torch.cuda.synchronize()
    finally:
        os.environ.pop("TREE_ATTN_TEST_STALL", None)
        os.environ["TREE_ATTN_CHECK"] = "1"
    code = int(p.status.item())
    assert code & kernels._lib.ERR_TIMEOUT, code
    assert not code & kernels._lib.ERR_BOUNDS, code
    p.status.zero_()
    lse = torch.empty(len(tree.paths), 8, device="cuda")
    out = attention_matrix(qd, kp, vp, p, out_lse=lse).cpu()
    torch.cuda.synchronize()
    check_status(p)
    check_against_oracle(q, k, v, tree.paths, out, lse.cpu())
