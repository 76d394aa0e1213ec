"""ta_attention_noalloc: the decode-step attention for callers that cannot allocate.

Some hosts cannot call cudaMalloc where they run attention (a process whose
device memory belongs to another allocator, a binding with no CUDA allocator, a
serving loop that must not allocate on its decode path).  This entry
point takes only inputs and outputs and keeps its scratch in a fixed device
array.  The test calls it through the C ABI twice in a row and checks both
results against the allocating entry point ta_attention on the same inputs.
It lives in its own file, collected last, and passes alone or after the rest.
"""
import pytest
import torch

from tree_attention import CostModel, KVTree, _lib, schedule
from tree_attention.kernels import pack_kv, prepare

pytestmark = pytest.mark.gpu

REL_L2 = 5e-3
LSE_TOL = 1e-3


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _inputs(seed=7):
    # a shared root (query-tile kernel) and private leaves (small-group kernel)
    tree = KVTree.synthetic([-1] + [0] * 48, [900] + [20 + i for i in range(48)], list(range(1, 49)))
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(48, 32, 128, generator=g).bfloat16().cuda()
    k = torch.randn(tree.storage_tokens, 8, 128, generator=g).bfloat16().cuda()
    v = torch.randn(tree.storage_tokens, 8, 128, generator=g).bfloat16().cuda()
    kp, vp = pack_kv(k, v)
    return tree, q, kp, vp


def _call(fn, p, q, kp, vp, out, lse, with_scratch):
    lib = _lib.load()
    args = [p.layout, p.metadata.data_ptr(), q.data_ptr(), kp.data_ptr(), vp.data_ptr(), kp.shape[1], 32, 8, 128,
            _lib.DTYPE_BF16]
    if with_scratch:
        args += [p.part.data_ptr(), p.lse.data_ptr()]
    args += [out.data_ptr(), lse.data_ptr(), p.status.data_ptr(), _stream()]
    return getattr(lib, fn)(*args)


def test_noalloc_matches_allocating_entry_point_twice():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    tree, q, kp, vp = _inputs()
    p = prepare(schedule(tree, method="cube", model=CostModel.b200()), q)
    assert p.layout.num_tc_tasks > 0 and p.layout.num_kn_tasks > 0
    ref_out = torch.empty_like(q)
    ref_lse = torch.empty(48, 32, device="cuda")
    assert _call("ta_attention", p, q, kp, vp, ref_out, ref_lse, True) == 0
    for _ in range(2):
        out = torch.full_like(q, float("nan"))
        lse = torch.full((48, 32), float("nan"), device="cuda")
        assert _call("ta_attention_noalloc", p, q, kp, vp, out, lse, False) == 0
        torch.cuda.synchronize()
        assert int(p.status.item()) == 0
        err = (out.float() - ref_out.float()).norm(dim=-1) / ref_out.float().norm(dim=-1)
        assert err.max().item() <= REL_L2
        assert (lse - ref_lse).abs().max().item() <= LSE_TOL


def test_noalloc_rejects_problems_beyond_its_scratch():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    # 32 KV heads x 2048 partial rows x 4 x 129 floats is far above 32 MiB
    tree = KVTree.synthetic([-1] + [0] * 2048, [8] + [1] * 2048, list(range(1, 2049)))
    q = torch.empty(2048, 128, 128, dtype=torch.bfloat16, device="cuda")
    kp = torch.empty(32, tree.storage_tokens, 128, dtype=torch.bfloat16, device="cuda")
    p = prepare(schedule(tree, 128, 32, 128, "fixed"), q)
    lib = _lib.load()
    rc = lib.ta_attention_noalloc(p.layout, p.metadata.data_ptr(), q.data_ptr(), kp.data_ptr(), kp.data_ptr(),
                                  kp.shape[1], 128, 32, 128, _lib.DTYPE_BF16, q.data_ptr(), None,
                                  p.status.data_ptr(), _stream())
    assert rc == _lib.ERR_TOO_LARGE
