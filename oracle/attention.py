"""TEST INFRASTRUCTURE ONLY -- FP32 CPU restatement of the reference's oracle.

Restates ``src/tree_attention/reference.py`` of Gxj230958/tree-attention-scheduling:

* ``request_attention`` (reference.py:4-13): for each request, full softmax
  attention of its query heads over the K/V rows on its path, GQA by repeating
  each KV head for ``G = HQ / HK`` query heads, scores scaled by ``D**-0.5``,
  everything in float32, output cast to the query dtype.
* ``segmented_attention`` (reference.py:16-33): per plan job, the partial
  output and the natural-log LSE of the job's scores; per request, the partials
  weighted by ``softmax`` over their LSEs.

Both also return the float32 output before the cast and the merged LSE, which
the reference does not expose; the LSE is ``logsumexp`` of the same scores
(reference.py:11 computes those scores).  Inputs use the reference layout:
``q [NREQ, HQ, D]``, ``k, v [T, HK, D]``.
"""
from __future__ import annotations

import torch


def _scores(qr, kr, dim):
    # qr [..., HQ, D], kr [n, HQ, D] -> [..., HQ, n]
    return torch.einsum("...hd,nhd->...hn", qr, kr) / dim ** 0.5


def request_attention(q, k, v, paths, return_lse=False):
    """Per-request FP32 attention (reference.py:4-13).

    ``paths``: the requests' token paths, or the ``KVTree`` itself (the
    reference's argument).  Returns the output in ``q.dtype``; with
    ``return_lse`` also the float32 output and the natural-log LSE ``[NREQ, HQ]``.
    """
    paths = getattr(paths, "paths", paths)
    groups = q.shape[1] // k.shape[1]
    dim = q.shape[-1]
    outs, lses = [], []
    for r, path in enumerate(paths):
        idx = torch.as_tensor(path, dtype=torch.long)
        kr = k.index_select(0, idx).float().repeat_interleave(groups, dim=1)
        vr = v.index_select(0, idx).float().repeat_interleave(groups, dim=1)
        s = _scores(q[r].float(), kr, dim)                    # [HQ, n]
        outs.append(torch.einsum("hn,nhd->hd", torch.softmax(s, -1), vr))
        lses.append(torch.logsumexp(s, -1))
    out = torch.stack(outs)
    if return_lse:
        return out.to(q.dtype), out, torch.stack(lses)
    return out.to(q.dtype)


def job_partials(q, k, v, jobs):
    """Partial output ``[|R|, HQ, D]`` and LSE ``[|R|, HQ]`` of every job (reference.py:20-27)."""
    groups = q.shape[1] // k.shape[1]
    dim = q.shape[-1]
    result = []
    for job in jobs:
        qs = q[list(job.requests)].float()
        idx = torch.as_tensor(job.tokens, dtype=torch.long)
        ks = k.index_select(0, idx).float().repeat_interleave(groups, 1)
        vs = v.index_select(0, idx).float().repeat_interleave(groups, 1)
        s = _scores(qs, ks, dim)                               # [|R|, HQ, n]
        result.append((torch.einsum("rhn,nhd->rhd", torch.softmax(s, -1), vs), torch.logsumexp(s, -1)))
    return result


def merge_partials(num_requests, jobs, partials):
    """Global LSE merge of per-request partials (reference.py:28-33)."""
    per_request = [[] for _ in range(num_requests)]
    for job, (out, lse) in zip(jobs, partials):
        for i, r in enumerate(job.requests):
            per_request[r].append((out[i], lse[i]))
    outs, lses = [], []
    for parts in per_request:
        o = torch.stack([p[0] for p in parts])                # [m, HQ, D]
        l = torch.stack([p[1] for p in parts])                # [m, HQ]
        outs.append((o * torch.softmax(l, 0)[..., None]).sum(0))
        lses.append(torch.logsumexp(l, 0))
    return torch.stack(outs), torch.stack(lses)


def segmented_attention(q, k, v, jobs, return_lse=False):
    """Plan-driven FP32 attention with the global LSE merge (reference.py:16-33).

    ``jobs``: the plan's jobs, or the ``Plan`` itself (the reference's argument).
    """
    jobs = getattr(jobs, "jobs", jobs)
    out, lse = merge_partials(q.shape[0], jobs, job_partials(q, k, v, jobs))
    if return_lse:
        return out.to(q.dtype), out, lse
    return out.to(q.dtype)
