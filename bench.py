"""Benchmark of the tree-shared decode-attention step on B200.

Workload (BASELINE headline, configs[1]): 128 requests, each with an 8192-token
context: a shared 8128-token root then 128 private 64-token leaves (16,320
physical / 1,048,576 logical KV positions); 32 query heads, 8 KV heads,
head_dim 128; Q/K/V BF16 drawn N(0,1) from a seed (synthetic data, no dataset);
one decode query per request; subset-DP ("cube") plan with the B200 cost model.

One step = one decode-step attention: the segment kernels over every
(job, KV head) plus the LSE merge, inputs resident in HBM.  Metric: physical-KV
HBM throughput (physical KV bytes / step time, GB/s, higher is better); the
step latency in microseconds is reported beside it.  The KV working set of one
step (66.8 MB) fits in the 126 MB L2, so consecutive steps rotate through
COPIES independent copies of the queries and pools (4 x 67 MB, larger than L2):
every step reads its KV from HBM, with no flush kernel in the timed region.
The K timed steps are one CUDA graph replay, timed with CUDA events.

With ``--gpus N`` (launched by torchrun, one process per GPU) the 8 KV heads are
sharded: rank r owns heads [r*8/N, (r+1)*8/N) with their query heads and that
slice of the pools; the plan is identical on every rank; no collective runs
inside attention.  Total work is fixed (strong scaling); the step time is the
max over ranks.

``--impl reference`` times the reference's CPU implementation of the path --
the FP32 plan-driven oracle (restated under ``oracle/``), all host threads --
on the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "tree-attention-scheduling_b200"))
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

# The package (and with it the kernel library) is imported by the GPU arms
# only: the reference arm runs nothing of this repository's engine.
CostModel = KVTree = schedule = kernels = _lib = None


def load_package():
    """Import tree_attention for the GPU arms (binds the module-level names)."""
    global CostModel, KVTree, schedule, kernels, _lib
    from tree_attention import CostModel, KVTree, schedule  # noqa: F811
    from tree_attention import kernels  # noqa: F811
    from tree_attention import _lib  # noqa: F811

METRIC = "tree-attn decode step µs & physical-KV HBM GB/s, 128req×8K ctx, 1–8 B200"
NREQ, ROOT_LEN, LEAF_LEN = 128, 8128, 64
HQ, HK, D = 32, 8, 128
SEED = 101
COPIES = 4
E2E_STEPS = 200          # steps per replay of the end-to-end loop
E2E_REPLAYS = 5          # replays timed; the median is reported
GRID_STEPS = 5           # steps per shape of the default line's grid summary
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0


def headline_tree():
    return KVTree.synthetic([-1] + [0] * NREQ, [ROOT_LEN] + [LEAF_LEN] * NREQ, list(range(1, NREQ + 1)))


def kv_bytes(tree, heads=HK):
    return tree.storage_tokens * heads * D * 2 * 2


def logical_flops(tree, q_heads=HQ):
    return 4 * D * q_heads * sum(len(p) for p in tree.paths)


def peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return data["hbm_gbs"], data["bf16_tflops"], "measured"
    return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, "fallback"


def profile_traffic():
    """Per-launch DRAM bytes of the segment phase from the committed ncu summary, if any."""
    path = ROOT / "profiles" / "seg_headline_traffic.txt"
    if not path.exists():
        return None
    for line in path.read_text().splitlines():
        if line.startswith("traffic_bytes_per_step:"):
            return int(line.split(":", 1)[1].strip())
    return None


def rank_traffic(local_heads):
    """DRAM bytes of one rank's segment phase: the one-GPU capture scaled by the rank's share of KV heads
    (every KV byte and partial row belongs to one head, so the traffic divides with the heads)."""
    full = profile_traffic()
    return None if full is None else int(round(full * local_heads / HK))


# ---------------------------------------------------------------------------
# inputs: every KV head (and its query heads) from its own generator, so the
# data are identical whatever the number of shards.
def make_inputs(tree, heads, device):
    storage = tree.storage_tokens
    G = HQ // HK
    q = torch.empty(NREQ, len(heads) * G, D, dtype=torch.bfloat16, device=device)
    kp = torch.empty(len(heads), storage, D, dtype=torch.bfloat16, device=device)
    vp = torch.empty_like(kp)
    for i, h in enumerate(heads):
        g = torch.Generator(device=device).manual_seed(SEED * 1000 + h)
        q[:, i * G:(i + 1) * G] = torch.randn(NREQ, G, D, generator=g, device=device).bfloat16()
        kp[i] = torch.randn(storage, D, generator=g, device=device).bfloat16()
        vp[i] = torch.randn(storage, D, generator=g, device=device).bfloat16()
    return q, kp, vp


class ClockSampler:
    """NVML sampler of SM clock and clock-event reasons (read-only)."""

    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
               0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}

    def __init__(self, index, period=0.005):
        self.samples, self.reasons = [], 0
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nvml = pynvml
            self._handle = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._handle, pynvml.NVML_CLOCK_SM)
        except Exception as exc:  # pragma: no cover - depends on the driver
            self._nvml = None
            self.error = repr(exc)
        self.period = period

    def _run(self):
        nv = self._nvml
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._handle, nv.NVML_CLOCK_SM))
                self.reasons |= nv.nvmlDeviceGetCurrentClocksEventReasons(self._handle)
            except Exception:
                pass
            time.sleep(self.period)

    def start(self):
        if self._nvml:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()

    def stop(self):
        if self._thread:
            self._stop.set()
            self._thread.join()
        names = sorted(n for bit, n in self.REASONS.items() if self.reasons & bit and n != "gpu_idle")
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": names, "samples": len(self.samples),
                "source": "nvml" if self._nvml else "unavailable"}


# ---------------------------------------------------------------------------
def setup_dist(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        if world == 1 and args.gpus > 1:
            raise SystemExit("--gpus N > 1 must be launched with torchrun (one process per GPU)")
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(local)
    return rank, world, local


def max_over_ranks(value, world):
    """The largest of every rank's `value` (device time of a multi-GPU step is the slowest rank's)."""
    if world == 1:
        return value
    import torch.distributed as dist
    device = "cpu" if dist.get_backend() == "gloo" else "cuda"
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()


class Step:
    """One decode step of a prepared plan over one of several input copies."""

    def __init__(self, copies, prepared):
        self.copies, self.p = copies, prepared
        self.q, self.kp, self.vp = copies[0]
        self.lib = _lib.load()
        L = prepared.layout
        small = sum(1 for i, e in enumerate(L.small_class_end) if e > (L.small_class_end[i - 1] if i else 0))
        kn = sum(1 for c in range(5) if L.kn_class_ctas[c] > 0)
        self.launches = small + (1 if L.num_tc_tasks else 0) + kn + 1          # + the merge

    def attention(self, copy=0):
        """The whole step through the public C entry point ta_attention."""
        p = self.p
        q, kp, vp = self.copies[copy]
        rc = self.lib.ta_attention(p.layout, p.metadata.data_ptr(), q.data_ptr(), kp.data_ptr(), vp.data_ptr(),
                                   kp.shape[1], q.shape[1], kp.shape[0], D, _lib.DTYPE_BF16, p.part.data_ptr(),
                                   p.lse.data_ptr(), p.out.data_ptr(), None, p.status.data_ptr(),
                                   torch.cuda.current_stream().cuda_stream)
        _lib.check(rc, "ta_attention")

    def segment(self, copy=0):
        p = self.p
        q, kp, vp = self.copies[copy]
        rc = self.lib.ta_segment(p.layout, p.metadata.data_ptr(), q.data_ptr(), kp.data_ptr(), vp.data_ptr(),
                                 kp.shape[1], q.shape[1], kp.shape[0], D, _lib.DTYPE_BF16, p.part.data_ptr(),
                                 p.lse.data_ptr(), p.status.data_ptr(), torch.cuda.current_stream().cuda_stream)
        _lib.check(rc, "ta_segment")

    def merge(self, copy=0):
        p = self.p
        rc = self.lib.ta_merge(p.layout, p.metadata.data_ptr(), p.part.data_ptr(), p.lse.data_ptr(),
                               p.out.data_ptr(), None, self.q.shape[1], self.kp.shape[0], D, _lib.DTYPE_BF16,
                               p.status.data_ptr(), torch.cuda.current_stream().cuda_stream)
        _lib.check(rc, "ta_merge")


def capture(fn):
    """Record fn's launches into a CUDA graph (after one eager warm call)."""
    fn()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.graph(graph, stream=stream):
        fn()
    torch.cuda.synchronize()
    return graph


def time_graph(graph, units, warmup, world):
    """Device microseconds per unit of one replay of `graph` (after `warmup` replays)."""
    for _ in range(warmup):
        graph.replay()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    graph.replay()
    e1.record()
    barrier(world)
    return e0.elapsed_time(e1) * 1e3 / units


def time_step(step, steps, warmup, world):
    """Device time (us) per step: K whole steps (ta_attention) in one graph, then the
    segment launches alone (ta_segment, for the per-kernel roofline) and the merge
    kernel alone, all rotating through the input copies so every step streams its
    KV from HBM."""
    n = len(step.copies)
    whole = capture(lambda: [step.attention(i % n) for i in range(steps)])
    step_us = time_graph(whole, steps, warmup, world)
    seg = capture(lambda: [step.segment(i % n) for i in range(steps)])
    seg_us = time_graph(seg, steps, warmup, world)
    merge = capture(lambda: [step.merge(i % n) for i in range(steps)])
    merge_us = time_graph(merge, steps, warmup, world)
    del whole, seg, merge
    return step_us, seg_us, merge_us


def time_e2e(q_host, plans, copies, steps, warmup, world):
    """Public-API decode loop with host buffers: every step copies its queries from pinned host memory,
    runs kernels.attention_matrix and copies the output back to pinned host memory.  The steps are
    pipelined over three streams, as a serving loop would run them: the H2D copy of step i+1 and the D2H
    copy of step i-1 overlap step i's attention.  Two plan objects alternate, so an output buffer is not
    rewritten before its copy to the host has finished.  The loop of K steps is timed twice: issued
    eagerly from Python, and recorded once into a CUDA graph and replayed (the serving-loop form: the
    Python work per step leaves the timed region, the copies and kernels stay).  The graph holds
    ``steps`` steps (at least E2E_STEPS) and is replayed E2E_REPLAYS times; the median replay is the
    figure.  Also returns each copy's time on its own."""
    n = len(copies)
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
    out_host = [torch.empty(p.out.shape, dtype=p.out.dtype, pin_memory=True) for p in plans]

    def run(count):
        comp = torch.cuda.current_stream()
        s_in.wait_stream(comp)
        s_out.wait_stream(comp)
        last_use = [None] * n            # compute event that last read each device copy of the queries
        out_free = [None] * len(plans)   # D2H event that last read each plan's output
        for i in range(count):
            c, b = i % n, i % len(plans)
            q_dev, kp, vp = copies[c]
            with torch.cuda.stream(s_in):
                if last_use[c] is not None:
                    s_in.wait_event(last_use[c])
                q_dev.copy_(q_host, non_blocking=True)
                landed = torch.cuda.Event()
                landed.record(s_in)
            comp.wait_event(landed)
            if out_free[b] is not None:
                comp.wait_event(out_free[b])
            out = kernels.attention_matrix(q_dev, kp, vp, plans[b])
            computed = torch.cuda.Event()
            computed.record(comp)
            last_use[c] = computed
            with torch.cuda.stream(s_out):
                s_out.wait_event(computed)
                out_host[b].copy_(out, non_blocking=True)
                copied = torch.cuda.Event()
                copied.record(s_out)
            out_free[b] = copied
        comp.wait_stream(s_in)
        comp.wait_stream(s_out)

    def timed(fn):
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        barrier(world)
        return e0.elapsed_time(e1) * 1e3 / steps

    run(warmup)
    eager_us = timed(lambda: run(steps))
    graph = capture(lambda: run(steps))
    graph.replay()
    replays = sorted(timed(graph.replay) for _ in range(E2E_REPLAYS))
    graph_us = replays[len(replays) // 2]
    del graph
    # one 1 MiB copy each way on its own: what the pipeline has to hide behind the kernels
    copy_us = []
    for dst, src in ((copies[0][0], q_host), (out_host[0], plans[0].out)):
        for _ in range(3):
            dst.copy_(src, non_blocking=True)
        copy_us.append(timed(lambda: [dst.copy_(src, non_blocking=True) for _ in range(steps)]))
    sizes = (q_host.numel() * q_host.element_size(), out_host[0].numel() * out_host[0].element_size())
    return dict(graph_us=graph_us, graph_replays_us=[round(x, 3) for x in replays], eager_us=eager_us,
                h2d_bytes=sizes[0], d2h_bytes=sizes[1], h2d_copy_us=copy_us[0], d2h_copy_us=copy_us[1])


def cpu_oracle_step_us(tree, plan, q, kp, vp, budget_s=10.0, max_steps=200):
    """The FP32 plan-driven oracle on the host cores, repeated for about budget_s seconds."""
    from oracle import attention as oracle
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    qc = q.float().cpu()
    kc = kp.float().cpu().permute(1, 0, 2).contiguous()
    vc = vp.float().cpu().permute(1, 0, 2).contiguous()
    oracle.segmented_attention(qc, kc, vc, plan.jobs)          # warm-up
    t0 = time.perf_counter()
    n = 0
    while n < max_steps and (n == 0 or time.perf_counter() - t0 < budget_s):
        oracle.segmented_attention(qc, kc, vc, plan.jobs)
        n += 1
    return (time.perf_counter() - t0) * 1e6 / n, n, threads


def run_b200(args):
    rank, world, local = setup_dist(args)
    if HK % world:
        raise SystemExit("the 8 KV heads must divide evenly over the GPUs")
    heads = list(range(rank * HK // world, (rank + 1) * HK // world))
    tree = headline_tree()
    dev = torch.device("cuda", local)
    q, kp, vp = make_inputs(tree, heads, dev)
    copies = [(q, kp, vp)] + [(q.clone(), kp.clone(), vp.clone()) for _ in range(COPIES - 1)]
    model = CostModel.b200()

    results = {}
    t0 = time.perf_counter()
    plan = schedule(tree, HQ, HK, D, args.method, model)
    plan_us = (time.perf_counter() - t0) * 1e6
    t0 = time.perf_counter()
    prepared = kernels.prepare(plan, q, num_kv_heads=len(heads))
    torch.cuda.synchronize()
    metadata_us = (time.perf_counter() - t0) * 1e6
    step = Step(copies, prepared)

    sampler = ClockSampler(local)
    sampler.start()
    burn_end = time.perf_counter() + (0.0 if args.quick else args.burn_s)
    i = 0
    while time.perf_counter() < burn_end:       # sustained load so the clock samples see the step
        step.attention(i % COPIES)
        i += 1
    step_us_local, seg_us, merge_us = time_step(step, args.steps, args.warmup, world)
    clocks = sampler.stop()
    kernels.check_status(prepared)
    step_us = max_over_ranks(step_us_local, world)
    seg_us_max = max_over_ranks(seg_us, world)

    # other plans on the same kernels (same shards), for the speed-up columns
    for method, m in (("request", CostModel()), ("fixed", model), ("greedy", model)):
        if args.quick or (not args.all_plans and method != "request"):
            continue
        pl = kernels.prepare(schedule(tree, HQ, HK, D, method, m), q, num_kv_heads=len(heads))
        whole, _, _ = time_step(Step(copies, pl), max(3, args.steps // 2), args.warmup, world)
        results[method] = {"step_us": max_over_ranks(whole, world), "jobs": len(pl.jobs)}
        del pl

    q_host = q.cpu().pin_memory()
    second = kernels.prepare(plan, q, num_kv_heads=len(heads))
    e2e = time_e2e(q_host, [prepared, second], copies, 20 if args.quick else max(E2E_STEPS, args.steps),
                   args.warmup, world)
    e2e_eager_us = max_over_ranks(e2e["eager_us"], world)
    kernels.check_status(second)
    del second
    e2e_us = max_over_ranks(e2e["graph_us"], world)
    h2d, d2h = e2e["h2d_bytes"], e2e["d2h_bytes"]
    kernels.check_status(prepared)

    total_bytes = kv_bytes(tree)                     # all ranks together
    local_bytes = kv_bytes(tree, len(heads))
    hbm_peak, tf_peak, peak_kind = peaks()
    achieved = local_bytes / (seg_us * 1e-6) / 1e9
    value = total_bytes / (step_us * 1e-6) / 1e9
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(step_us / 1e3, 6), "step_us": round(step_us, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) BF16 Q/K/V)",
        "config": {"workload": "headline: 128 req x 8192 ctx, shared 8128-token root + 128 x 64-token leaves, "
                               "HQ=32 HK=8 D=128, one decode query per request",
                   "plan": args.method, "cost_model": "CostModel.b200()", "jobs": len(prepared.jobs),
                   "physical_kv_bytes": total_bytes, "logical_kv_bytes": sum(len(p) for p in tree.paths) * HK * D * 4,
                   "parallelism": f"kv-head shard x{world}" if world > 1 else "single GPU",
                   "l2": f"inputs larger than L2: steps rotate through {COPIES} copies of Q/K/V "
                         f"({COPIES} x {kv_bytes(tree, len(heads)) / 1e6:.1f} MB)",
                   "timing": "CUDA events around one CUDA-graph replay of K consecutive steps",
                   "plan_us": round(plan_us, 1), "metadata_us": round(metadata_us, 1)},
        "segment_us": round(seg_us_max, 3), "merge_us": round(max_over_ranks(merge_us, world), 3),
        "e2e": {"value": round(total_bytes / (e2e_us * 1e-6) / 1e9, 2), "unit": "GB/s", "step_us": round(e2e_us, 3),
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "path": "kernels.attention_matrix per step with pinned host Q in and output out, steps pipelined "
                        "over three streams (H2D of step i+1 and D2H of step i-1 overlap step i); the loop of "
                        f"{E2E_STEPS} steps recorded once as a CUDA graph, median of {E2E_REPLAYS} replays",
                "replays_us": e2e["graph_replays_us"], "eager_step_us": round(e2e_eager_us, 3),
                "h2d_copy_us": round(e2e["h2d_copy_us"], 2), "d2h_copy_us": round(e2e["d2h_copy_us"], 2)},
        "gpu_launches": step.launches * args.steps,
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                     "frac": round(achieved / hbm_peak, 4), "traffic": rank_traffic(len(heads)),
                     "kernel": "segment phase (all segment launches of one step)",
                     "peak_source": f"{peak_kind} hbm_gbs",
                     "tensor_tflops": round(logical_flops(tree, HQ * len(heads) // HK) / (seg_us * 1e-6) / 1e12, 1),
                     "tensor_frac": round(logical_flops(tree, HQ * len(heads) // HK) / (seg_us * 1e-6) / 1e12 /
                                          tf_peak, 4)},
        "clocks": clocks,
        "plans": results,
    }
    if "request" in results:
        line["per_request_speedup"] = round(results["request"]["step_us"] / step_us, 3)
    if world == 1 and rank == 0 and not (args.no_cpu_baseline or args.quick):
        cpu_us, n, threads = cpu_oracle_step_us(tree, plan, q, kp, vp, budget_s=args.cpu_budget_s)
        line["cpu_baseline"] = {"value": round(total_bytes / (cpu_us * 1e-6) / 1e9, 4), "unit": "GB/s",
                                "step_us": round(cpu_us, 1), "cores": threads, "kind": "port",
                                "sample": f"{n} full headline steps of the FP32 plan-driven oracle "
                                          f"(oracle/attention.py segmented_attention, same cube plan)"}
    if world == 1 and not (args.quick or args.no_extras):
        # the other BASELINE configurations, compactly: configs[2] (every grid shape, few steps) and
        # configs[3] (the cube plan reused vs rebuilt)
        geo, rows = grid_summary(GRID_STEPS, 3)
        speedups = [r["speedup"] for r in rows]
        line["grid"] = {"geomean_speedup": round(geo, 4), "min": min(speedups), "max": max(speedups),
                        "shapes": len(rows), "steps": GRID_STEPS, "target": 1.3,
                        "what": "configs[2]: tree (cube) plan vs per-request plan on the same kernels"}
        rows = {r["mode"]: r for r in decode_summary(("cube",))}
        line["decode_reuse"] = {"cached_step_us": rows["cached"]["per_step_us"],
                                "rebuilt_step_us": rows["rebuild"]["per_step_us"],
                                "cached_attention_us": rows["cached"]["attention_us"],
                                "cached_planning_us": rows["cached"]["planning_us"],
                                "rebuilt_planning_us": rows["rebuild"]["planning_us"],
                                "max_rel_l2": max(rows["cached"]["max_rel_l2"], rows["rebuild"]["max_rel_l2"]),
                                "what": "configs[3], cube plan: planning + attention per decode step"}
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


class _Job:
    """A job of the reference's plan: requests and physical token positions."""

    def __init__(self, requests, runs):
        self.requests = tuple(requests)
        self.tokens = tuple(t for start, length in runs for t in range(start, start + length))


def reference_headline_jobs():
    """The reference's own cube plan of the headline tree (its default cost model), as recorded from the
    reference itself in tests/golden/headline_plan.json."""
    data = json.loads((ROOT / "tests" / "golden" / "headline_plan.json").read_text())
    return [_Job(r, runs) for r, runs in data["jobs"]], data


def run_reference(args):
    """The reference's CPU implementation of the path (FP32 oracle port), rank 0 only.

    It plans with the reference's own scheduler and cost model (the plan the reference itself produced
    for this tree, read from a committed fixture) and runs the plan-driven FP32 oracle on all host
    threads; nothing of this repository's package or kernel library is imported.
    """
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import attention as oracle
    jobs, recorded = reference_headline_jobs()
    storage = ROOT_LEN + NREQ * LEAF_LEN
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(SEED)
    q = torch.randn(NREQ, HQ, D, generator=g).bfloat16().float()
    k = torch.randn(storage, HK, D, generator=g).bfloat16().float()
    v = torch.randn(storage, HK, D, generator=g).bfloat16().float()
    for _ in range(args.warmup):
        oracle.segmented_attention(q, k, v, jobs)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        oracle.segmented_attention(q, k, v, jobs)
    us = (time.perf_counter() - t0) * 1e6 / args.steps
    value = storage * HK * D * 4 / (us * 1e-6) / 1e9
    line = {"impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "GB/s", "n_gpus": 0,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(us / 1e3, 3), "step_us": round(us, 1),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded N(0,1) BF16-valued Q/K/V)",
            "config": {"workload": "headline: 128 req x 8192 ctx, shared 8128-token root + 128 x 64-token leaves, "
                                   "HQ=32 HK=8 D=128", "plan": "cube",
                       "cost_model": "CostModel() (the reference's defaults)", "jobs": len(jobs),
                       "plan_source": "the reference's own schedule() output, tests/golden/headline_plan.json "
                                      f"(sha256 {recorded['digest'][:16]})"},
            "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": threads, "kind": "port",
                             "sample": f"{args.steps} full headline steps of the FP32 plan-driven oracle "
                                       "(oracle/attention.py segmented_attention) on the reference's plan"},
            "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# Other BASELINE configurations (run explicitly; the default line is the headline)
def random_inputs(tree, nreq, device, seed, copies=1):
    g = torch.Generator(device=device).manual_seed(seed)
    out = []
    for _ in range(copies):
        q = torch.randn(nreq, HQ, D, generator=g, device=device).bfloat16()
        kp = torch.randn(HK, tree.storage_tokens, D, generator=g, device=device).bfloat16()
        vp = torch.randn(HK, tree.storage_tokens, D, generator=g, device=device).bfloat16()
        out.append((q, kp, vp))
    return out


def grid_summary(steps, warmup, seed=201):
    """every shape of the 81-shape evaluation grid, tree (cube) plan vs per-request plan on the
    same kernels.  Returns (geomean speed-up, rows)."""
    from tree_attention import workloads
    import math
    model = CostModel.b200()
    rows = []
    for params, tree in workloads.evaluation_grid(seed=seed):
        nreq = len(tree.paths)
        kvb = kv_bytes(tree)
        copies = max(1, min(8, math.ceil((256 << 20) / kvb)))
        inputs = random_inputs(tree, nreq, "cuda", 201, copies)
        row = dict(params, storage_tokens=tree.storage_tokens, logical_tokens=sum(map(len, tree.paths)))
        for method in ("cube", "request"):
            t0 = time.perf_counter()
            plan = schedule(tree, HQ, HK, D, method, model)
            plan_us = (time.perf_counter() - t0) * 1e6
            prepared = kernels.prepare(plan, inputs[0][0])
            step = Step(inputs, prepared)
            whole, _, _ = time_step(step, steps, warmup, 1)
            kernels.check_status(prepared)
            row[method] = dict(step_us=round(whole, 2), plan_us=round(plan_us, 1), jobs=len(prepared.jobs))
            del prepared, step
        row["speedup"] = round(row["request"]["step_us"] / row["cube"]["step_us"], 4)
        rows.append(row)
        del inputs
        torch.cuda.empty_cache()
    speedups = [r["speedup"] for r in rows]
    return math.exp(sum(math.log(x) for x in speedups) / len(speedups)), rows


def run_grid(args):
    """81 seeded shapes, tree plan vs per-request plan on the same kernels."""
    torch.cuda.set_device(0)
    geo, rows = grid_summary(args.steps, args.warmup, args.seed or 201)
    speedups = [r["speedup"] for r in rows]
    line = {"config": "grid (configs[2]): 81 shapes, requests {16,64,256} x depth {1,2,4} x shared "
                      "{0.25,0.75,0.99} x branching {2,4,16}, context 2048-16384",
            "metric": "geomean speed-up of the tree (cube) plan over the per-request plan, same kernels",
            "value": round(geo, 4), "min": min(speedups), "max": max(speedups), "shapes": len(rows),
            "steps": args.steps, "warmup": args.warmup, "cost_model": "CostModel.b200()", "rows": rows}
    print(json.dumps(line), flush=True)


def run_calibrate(args):
    """Fit CostModel.b200()'s constants on the calibration grid (disjoint from the evaluation grid)."""
    from tree_attention import calibration, workloads
    import math
    torch.cuda.set_device(0)
    trees, inputs = [], []
    for index, (params, tree) in enumerate(workloads.calibration_grid()):
        copies = max(1, min(8, math.ceil((256 << 20) / kv_bytes(tree))))
        trees.append(tree)
        inputs.append(random_inputs(tree, len(tree.paths), "cuda", 501 + index, copies))
    position = {id(t): i for i, t in enumerate(trees)}
    steps, warmup = max(3, args.steps), max(3, args.warmup)

    def measure(model, tree):
        copies = inputs[position[id(tree)]]
        prepared = kernels.prepare(schedule(tree, HQ, HK, D, "cube", model), copies[0][0])
        step = Step(copies, prepared)
        n = len(copies)
        graph = capture(lambda: [step.attention(i % n) for i in range(steps)])
        us = time_graph(graph, steps, warmup, 1)
        kernels.check_status(prepared)
        del graph, step, prepared
        return us

    t0 = time.perf_counter()
    best, score, history = calibration.fit(trees, measure, log=lambda h: print(json.dumps(h), file=sys.stderr,
                                                                             flush=True))
    start = history[0]["geomean_us"]
    line = {"config": "calibrate: cost-model constants fitted on workloads.calibration_grid() (24 trees)",
            "metric": "geomean decode-step time over the calibration trees (us)",
            "start": start, "fitted": round(score, 3), "constants": best, "evaluated": len(history),
            "seconds": round(time.perf_counter() - t0, 1), "steps": steps, "warmup": warmup}
    print(json.dumps(line), flush=True)


def run_qwen(args):
    """random-init Qwen3-4B, 16 requests sharing a 3000-token document + 64 private tokens each,
    greedy decode with cached tree plans (CachedPrefixDecoder), KV heads sharded over the launched GPUs."""
    from transformers import Qwen3Config, Qwen3ForCausalLM
    from tree_attention import qwen
    rank, world, local = setup_dist(args)
    steps = args.steps if args.steps != 20 else 64
    config = Qwen3Config(vocab_size=151936, hidden_size=2560, intermediate_size=9728, num_hidden_layers=36,
                         num_attention_heads=32, num_key_value_heads=8, head_dim=128, rope_theta=1_000_000.0,
                         rms_norm_eps=1e-6, max_position_embeddings=8192, tie_word_embeddings=True,
                         initializer_range=0.02, attn_implementation="eager")
    torch.manual_seed(401)
    with torch.device("cuda", local):
        model = Qwen3ForCausalLM(config).to(torch.bfloat16).eval()
    g = torch.Generator().manual_seed(401)
    document = torch.randint(0, config.vocab_size, (3000,), generator=g).tolist()
    sequences = [document + torch.randint(0, config.vocab_size, (64,), generator=g).tolist() for _ in range(16)]
    group = None
    if world > 1:
        import torch.distributed as dist
        group = dist.group.WORLD
    results = {}
    for method, cost in (("cube", CostModel.b200()), ("request", CostModel())):
        barrier(world)
        t0 = time.perf_counter()
        eager_steps = 8
        decoder = qwen.CachedPrefixDecoder(model, sequences, max_new_tokens=steps + args.warmup + eager_steps + 1,
                                           method=method,
                                           cost_model=cost, shard=(rank, world, group) if world > 1 else None)
        torch.cuda.synchronize()
        prefill_s = time.perf_counter() - t0
        for _ in range(args.warmup):
            decoder.step(decoder.logits.argmax(-1).tolist())
        # eager Python step loop (one host read of the argmax per step)
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(eager_steps):
            decoder.step(decoder.logits.argmax(-1).tolist())
        e1.record()
        barrier(world)
        eager_ms = max_over_ranks(e0.elapsed_time(e1) / eager_steps, world)
        # the decode step recorded once as a CUDA graph and replayed (device-side greedy loop).  Each
        # generate() call captures its own graph and runs one eager warm-up step first; the per-step
        # figure is timed around the replays alone (events recorded inside generate), the whole call
        # (capture included) is reported beside it.
        r0, r1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

        def timed_generate(n):
            barrier(world)
            e0.record()
            decoder.generate(n, events=(r0, r1))
            e1.record()
            barrier(world)
            return (max_over_ranks(e0.elapsed_time(e1), world),
                    max_over_ranks(r0.elapsed_time(r1) / n, world))
        one_ms, _ = timed_generate(1)
        all_ms, ms = timed_generate(steps)
        results[method] = {"ms_per_step": round(ms, 3), "tokens_per_s": round(16 * 1000.0 / ms, 1),
                           "ms_per_step_incl_capture": round(all_ms / steps, 3),
                           "capture_and_first_step_ms": round(one_ms, 1),
                           "eager_ms_per_step": round(eager_ms, 3), "prefill_s": round(prefill_s, 2),
                           "pool_tokens": decoder.prefix_size, "jobs": len(decoder.cached_plan.prepared.jobs)}
        del decoder
        torch.cuda.empty_cache()
    line = {"config": "qwen (configs[4]): random-init Qwen3-4B (36 layers, hidden 2560, 32/8 heads, d 128, "
                      "SwiGLU 9728, vocab 151936, bf16, N(0, 0.02)), 16 requests x (3000 shared + 64 private) "
                      "uniform-random tokens, greedy decode with cached tree plans",
            "metric": "decode step latency (ms) and generated tokens/s, whole model (graph-replayed step; the "
                      "eager Python step loop beside it)", "n_gpus": world,
            "steps": steps, "warmup": args.warmup, "parallelism": f"kv-head shard x{world}" if world > 1 else
            "single GPU", "results": results,
            "tree_vs_request": round(results["request"]["ms_per_step"] / results["cube"]["ms_per_step"], 3)}
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


def decode_summary(methods=("fixed", "greedy", "cube")):
    """a 32-request 2-level tree, 16 decode steps of one token per request; the plan built once
    at prompt time and reused (CachedDecodePlan) vs rebuilt every step.  One row per (method, mode) with
    planning + attention per step; the first and last steps are checked against the FP32 oracle."""
    from tree_attention import workloads
    from tree_attention.kernels import CachedDecodePlan
    from oracle import attention as oracle
    import copy as _copy
    steps = 16
    base = workloads.decode_tree()
    prefix = base.storage_tokens
    nreq = len(base.paths)
    g = torch.Generator(device="cuda").manual_seed(301)
    q = torch.randn(nreq, HQ, D, generator=g, device="cuda").bfloat16()
    kp = torch.randn(HK, prefix + nreq * steps, D, generator=g, device="cuda").bfloat16()
    vp = torch.randn_like(kp)
    model = CostModel.b200()
    results = []

    def device_us(fn, reps=10):
        # reps back-to-back calls recorded in one CUDA graph: device time without launch gaps
        graph = capture(lambda: [fn() for _ in range(reps)])
        t = time_graph(graph, reps, 2, 1)
        del graph
        return t

    def check(step, out):
        paths = [path + tuple(prefix + r * steps + t for t in range(step + 1)) for r, path in enumerate(base.paths)]
        sample = [0, nreq // 2, nreq - 1]
        _, ref, _ = oracle.request_attention(q[sample].float().cpu(), kp.permute(1, 0, 2).float().cpu(),
                                             vp.permute(1, 0, 2).float().cpu(), [paths[r] for r in sample],
                                             return_lse=True)
        err = ((out[sample].float().cpu() - ref).norm(dim=-1) / ref.norm(dim=-1)).max().item()
        if err > 5e-3:
            raise AssertionError(f"decode step {step}: rel L2 {err:.3e}")
        return err

    for method in methods:
        for mode in ("rebuild", "cached"):
            tree = _copy.deepcopy(base)
            leaves = list(range(len(base.nodes) - nreq, len(base.nodes)))
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            cached = CachedDecodePlan(schedule(tree, HQ, HK, D, method, model), q, prefix, steps) \
                if mode == "cached" else None
            torch.cuda.synchronize()
            initial_us = (time.perf_counter() - t0) * 1e6
            per_step, worst = [], 0.0
            for step in range(steps):
                torch.cuda.synchronize()
                t0 = time.perf_counter()
                if mode == "rebuild":
                    tree.extend_leaves(leaves, [prefix + r * steps + step for r in range(nreq)])
                    p = kernels.prepare(schedule(tree, HQ, HK, D, method, model), q)
                else:
                    p = cached.update(step + 1)
                torch.cuda.synchronize()
                planning_us = (time.perf_counter() - t0) * 1e6
                att_us = device_us(lambda: kernels.attention_matrix(q, kp, vp, p))
                kernels.check_status(p)
                if step in (0, steps - 1):
                    worst = max(worst, check(step, kernels.attention_matrix(q, kp, vp, p).clone()))
                per_step.append(dict(step=step + 1, planning_us=round(planning_us, 1), attention_us=round(att_us, 2)))
            total = [s["planning_us"] + s["attention_us"] for s in per_step]
            results.append(dict(method=method, mode=mode, initial_plan_us=round(initial_us, 1),
                                planning_us=round(sum(s["planning_us"] for s in per_step) / steps, 1),
                                attention_us=round(sum(s["attention_us"] for s in per_step) / steps, 2),
                                per_step_us=round(sum(total) / steps, 1),
                                amortized_us=round((initial_us + sum(total)) / steps, 1),
                                max_rel_l2=worst))
    return results


def run_decode(args):
    """a 32-request 2-level tree, 16 decode steps, plan reused vs rebuilt."""
    torch.cuda.set_device(0)
    line = {"config": "decode (configs[3]): 32 requests, 4096-token root, 4 x 1024 branches, 32 x 256 leaves, "
                      "16 steps of 1 token per request", "metric": "planning + attention per step (us)",
            "cost_model": "CostModel.b200()", "results": decode_summary()}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--method", default="cube", choices=["request", "fixed", "greedy", "cube"])
    ap.add_argument("--all-plans", action="store_true", help="also time the fixed and greedy plans")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true", help="skip the grid and decode-reuse summaries")
    ap.add_argument("--cpu-budget-s", type=float, default=10.0)
    ap.add_argument("--burn-s", type=float, default=1.0, help="sustained untimed load before timing (clocks)")
    ap.add_argument("--config", choices=["headline", "grid", "decode", "calibrate", "qwen"], default="headline")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--quick", action="store_true",
                    help="main plan only: no burn, other plans, CPU baseline or repeated e2e (profiling runs)")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be at least 3")
    if args.impl == "reference":
        run_reference(args)
        return
    load_package()
    if args.config == "grid":
        run_grid(args)
    elif args.config == "decode":
        run_decode(args)
    elif args.config == "calibrate":
        run_calibrate(args)
    elif args.config == "qwen":
        run_qwen(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
