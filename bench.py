"""Benchmark of the sm_100a BF16 causal attention forward (prefill + KV-cache decode).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload W]

Headline line (``--workload prefill``, default): BASELINE config 3, causal prefill
B=4 H=12 Tq=Tk=4096 D=64 BF16 N(0,1), one step = one forward call; metric TFLOP/s over the
visible (i, j) pairs (4*B*H*D*T(T+1)/2 FLOP). The same line carries a ``decode`` block for
BASELINE config 4 (B=64 H=12 Tk=8192 decode, per-sequence lengths U[1024, 8192] by seed),
metric GB/s of the visible K/V rows plus q, O and LSE. ``--workload decode`` prints the decode
measurement as the headline instead; ``--workload generation`` times BASELINE config 5 (greedy
generation through a random-init decoder, TTFT / TPOT / tokens per second per attention
backend).

Multi-GPU (torchrun, one process per GPU): each rank owns an independent shard of the same shape
(weak scaling: the (batch x head) work of prefill and the batch of decode partition without any
exchange), timing is the max over ranks, ``value`` is the whole-job aggregate.

``--impl reference`` times the CPU oracle (a numpy restatement of the reference's
``reference.attention``, oracle/attention_oracle.py) on the host cores on a bounded sample of the
same workload; under torchrun only rank 0 runs it.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PREFILL_CFG = dict(B=4, H=12, T=4096, D=64)
DECODE_CFG = dict(B=64, H=12, Tk=8192, D=64, len_lo=1024, len_hi=8192, seed=2026)
L2_FLUSH_BYTES = 256 << 20  # > 126 MB L2
E2E_SLICES = 8  # (batch, head) row slices of the overlapped host-buffer e2e call


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return {"hbm_gbs": p["hbm_gbs"], "bf16_tflops": p["bf16_tflops"],
                "bf16_tflops_sustained": p.get("bf16_tflops_sustained"), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


def load_traffic():
    """Per-launch DRAM bytes of the dominant kernels from the committed ncu summaries
    (profiles/traffic.txt: `<kernel> <bytes per launch>` lines), or {} when absent."""
    path = os.path.join(ROOT, "profiles", "traffic.txt")
    out = {}
    if os.path.exists(path):
        for line in open(path):
            parts = line.split("#")[0].split()
            if len(parts) == 2:
                out[parts[0]] = float(parts[1])
    return out


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.file = None

    def __enter__(self):
        try:
            self.file = tempfile.TemporaryFile(mode="w+")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.file, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if self.proc is None or self.file is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.file.seek(0)
        rows = [r.split(", ") for r in self.file.read().strip().splitlines() if r.count(",") >= 8]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        mhz, mx, reasons = [], None, set()
        for r in rows:
            try:
                mhz.append(float(r[1]))
                mx = float(r[2])
            except ValueError:
                continue
            for name, val in zip(names, r[5:9]):
                if val.strip().lower() == "active":
                    reasons.add(name)
        if not mhz:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": 0}
        busy = [m for m in mhz if m >= 0.5 * max(mhz)]
        return {"sm_mhz": statistics.median(busy), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(mhz)}


# ----------------------------------------------------------------------------- distributed
def init_dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def reduce_max(value, world):
    if world == 1:
        return value
    import torch
    import torch.distributed as dist
    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


# ----------------------------------------------------------------------------- workloads
def decode_lengths(cfg, rank):
    rng = np.random.default_rng(cfg["seed"] + rank)
    return rng.integers(cfg["len_lo"], cfg["len_hi"] + 1, size=cfg["B"]).astype(np.int32)


def make_prefill(torch, rank):
    c = PREFILL_CFG
    g = torch.Generator(device="cuda").manual_seed(1000 + rank)
    shape = (c["B"], c["H"], c["T"], c["D"])
    q, k, v = [torch.randn(shape, generator=g, device="cuda", dtype=torch.bfloat16) for _ in range(3)]
    return q, k, v


def make_decode(torch, rank):
    c = DECODE_CFG
    g = torch.Generator(device="cuda").manual_seed(2000 + rank)
    q = torch.randn((c["B"], c["H"], 1, c["D"]), generator=g, device="cuda", dtype=torch.bfloat16)
    k = torch.randn((c["B"], c["H"], c["Tk"], c["D"]), generator=g, device="cuda", dtype=torch.bfloat16)
    v = torch.randn_like(k)
    lens = torch.from_numpy(decode_lengths(c, rank)).cuda()
    return q, k, v, lens


def time_device(torch, fn, steps, warmup, flush=None):
    """CUDA-event time of `fn` per step (ms list) on the current stream; `flush` runs between
    steps, outside the events."""
    for _ in range(warmup):
        fn()
        if flush is not None:
            flush()
    torch.cuda.synchronize()
    times = []
    for _ in range(steps):
        if flush is not None:
            flush()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        b.synchronize()
        times.append(a.elapsed_time(b))
    return times


def run_ours(args):
    import torch
    world, rank, local = init_dist()
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    import __graft_entry__
    __graft_entry__.import_package()
    from tiny_transformer_b200.operators import student
    from tiny_transformer_b200.operators.host_stream import attention_from_host
    from tiny_transformer_b200.operators._extension import load_attention_extension
    from oracle import attention_oracle as oracle
    ext = load_attention_extension()
    peaks = load_peaks()
    traffic = load_traffic()
    flush_buf = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device="cuda")

    def flush():
        flush_buf.fill_(1)

    def busy():
        # A ~50 us spin kernel with no memory traffic: the GPU is still busy while the host
        # enqueues the timed step, so host launch latency stays outside the events.
        torch.cuda._sleep(100_000)

    results = {}
    with torch.no_grad():
        # ------------------------------------------------------------------ prefill (cfg 3)
        c = PREFILL_CFG
        q, k, v = make_prefill(torch, rank)
        flops = oracle.prefill_flops(c["B"], c["H"], c["T"], c["T"], 0)
        fn = lambda: ext.attention_forward(q, k, v, 0)  # noqa: E731
        barrier(world)
        torch.cuda.synchronize()
        with ClockSampler(local) as clk:
            times = time_device(torch, fn, args.steps, args.warmup, flush)
            barrier(world)
            torch.cuda.synchronize()
        kernel_ms = sum(times) / len(times)
        step_ms = reduce_max(kernel_ms, world)
        # SDPA (FlashAttention backend) on the same GPU and inputs, for context.
        sd = lambda: torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=True)  # noqa: E731
        sdpa_ms = sum(time_device(torch, sd, max(3, args.steps // 2), args.warmup, flush)) / max(3, args.steps // 2)
        # end to end through the public operator: pinned host -> device, call, device -> host
        hq, hk, hv = [x.cpu().pin_memory() for x in (q, k, v)]
        ho = torch.empty(q.shape, dtype=torch.bfloat16, pin_memory=True)
        hl = torch.empty(q.shape[:-1], dtype=torch.float32, pin_memory=True)

        def e2e_serial():
            dq, dk, dv = [h.to("cuda", non_blocking=True) for h in (hq, hk, hv)]
            o, lse = student.attention_with_lse(dq, dk, dv, 0)
            ho.copy_(o, non_blocking=True)
            hl.copy_(lse, non_blocking=True)

        def e2e():
            # The same copies and kernel, sliced by (batch, head) rows so that input copies,
            # kernels and output copies overlap on three streams.
            attention_from_host(hq, hk, hv, 0, out=ho, lse=hl, slices=E2E_SLICES)
        e2e_steps = max(3, args.steps // 2)
        e2e_ms = reduce_max(sum(time_device(torch, e2e, e2e_steps, 2)) / e2e_steps, world)
        serial_ms = reduce_max(sum(time_device(torch, e2e_serial, e2e_steps, 2)) / e2e_steps, world)
        h2d = sum(x.numel() * x.element_size() for x in (hq, hk, hv))
        d2h = ho.numel() * 2 + hl.numel() * 4
        achieved = flops / (kernel_ms * 1e-3) / 1e12
        tr = traffic.get("attention_prefill_kernel")
        results["prefill"] = {
            "metric": "causal attn fwd TFLOP/s (prefill)",
            "value": round(world * flops / (step_ms * 1e-3) / 1e12, 2),
            "unit": "TFLOP/s",
            "ms_per_step": round(step_ms, 4),
            "config": {"workload": "cfg3 causal prefill B=4 H=12 Tq=Tk=4096 D=64 bf16 N(0,1), per rank",
                       "global_batch": c["B"] * world, "heads": c["H"], "seq_len": c["T"],
                       "head_dim": c["D"], "parallelism": f"(batch x head) shards, {world} rank(s)",
                       "l2": "flushed between timed steps (256 MiB write)"},
            "roofline": {"bound": "tensor", "achieved": round(achieved, 2),
                         "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": round(achieved / peaks["bf16_tflops"], 4),
                         "peak_kind": f"{peaks['source']} burst cuBLAS bf16",
                         "traffic": tr, "algorithmic_flops": flops},
            "e2e": {"value": round(world * flops / (e2e_ms * 1e-3) / 1e12, 3), "unit": "TFLOP/s",
                    "ms_per_step": round(e2e_ms, 3), "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h,
                    "api": f"operators.host_stream.attention_from_host, {E2E_SLICES} slices",
                    "serial": {"value": round(world * flops / (serial_ms * 1e-3) / 1e12, 3),
                               "ms_per_step": round(serial_ms, 3),
                               "api": "copy in, student.attention_with_lse, copy out"}},
            "gpu_launches": args.steps,
            "sdpa": {"value": round(flops / (sdpa_ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
                     "ms_per_step": round(sdpa_ms, 4)},
            "clocks": clk.summary(),
        }
        del hq, hk, hv, ho, hl

        # ------------------------------------------------------------------ backward (cfg 3)
        # dQ, dK, dV of the same prefill (the training path of student.attention); work counted
        # as 2.5x the forward FLOPs (five GEMMs: QK^T recomputed, dO.V^T, P^T.dO, dS^T.Q, dS.K).
        out, lse = ext.attention_forward(q, k, v, 0)
        g = torch.Generator(device="cuda").manual_seed(77 + rank)
        dout = torch.randn(q.shape, device="cuda", dtype=torch.bfloat16, generator=g)
        bwd_flops = 2.5 * flops
        bsteps = max(3, args.steps // 2)
        fn = lambda: ext.attention_backward(q, k, v, dout, out, lse, 0)  # noqa: E731
        barrier(world)
        torch.cuda.synchronize()
        times = time_device(torch, fn, bsteps, args.warmup, flush)
        barrier(world)
        torch.cuda.synchronize()
        bwd_ms = reduce_max(sum(times) / len(times), world)
        # The fixed-order path taken under torch.use_deterministic_algorithms(True) (this rank).
        det_mode = (torch.are_deterministic_algorithms_enabled(),
                    torch.is_deterministic_algorithms_warn_only_enabled())
        torch.use_deterministic_algorithms(True)
        try:
            det_ms = sum(time_device(torch, fn, bsteps, args.warmup, flush)) / bsteps
        finally:
            torch.use_deterministic_algorithms(det_mode[0], warn_only=det_mode[1])
        with torch.enable_grad():
            qq, kk, vv = [x.detach().requires_grad_() for x in (q, k, v)]
            o2 = torch.nn.functional.scaled_dot_product_attention(qq, kk, vv, is_causal=True)
            sd = lambda: torch.autograd.grad(o2, (qq, kk, vv), dout, retain_graph=True)  # noqa: E731
            sdpa_bwd_ms = sum(time_device(torch, sd, bsteps, args.warmup, flush)) / bsteps
            del qq, kk, vv, o2
        results["backward"] = {
            "metric": "causal attn bwd TFLOP/s (2.5x forward FLOPs)",
            "value": round(world * bwd_flops / (bwd_ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
            "ms_per_step": round(bwd_ms, 4),
            "config": {"workload": "cfg3 backward (dQ, dK, dV) B=4 H=12 Tq=Tk=4096 D=64 bf16, "
                                   "per rank", "algorithmic_flops": bwd_flops},
            "roofline": {"bound": "tensor",
                         "achieved": round(bwd_flops / (bwd_ms * 1e-3) / 1e12, 2),
                         "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": round(bwd_flops / (bwd_ms * 1e-3) / 1e12 / peaks["bf16_tflops"], 4)},
            "gpu_launches": 3 * bsteps,
            "sdpa": {"value": round(bwd_flops / (sdpa_bwd_ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
                     "ms_per_step": round(sdpa_bwd_ms, 4)},
            "deterministic": {"value": round(bwd_flops / (det_ms * 1e-3) / 1e12, 2),
                              "unit": "TFLOP/s", "ms_per_step": round(det_ms, 4)},
        }
        del q, k, v, out, lse, dout

        # ------------------------------------------------------------------ decode (cfg 4)
        c = DECODE_CFG
        q, k, v, lens = make_decode(torch, rank)
        lens_np = lens.cpu().numpy()
        nbytes = oracle.decode_bytes(c["B"], c["H"], lens_np)
        fn = lambda: ext.attention_forward(q, k, v, c["Tk"] - 1, None, lens)  # noqa: E731
        barrier(world)
        torch.cuda.synchronize()
        # The K/V read (~0.9 GB) is 7x L2, so the headline uses no flush: a 256 MiB flush write
        # leaves up to L2's worth of dirty lines whose write-back would land inside the timed
        # step. The flushed timing is reported beside it.
        with ClockSampler(local) as clk:
            times = time_device(torch, fn, args.steps, args.warmup, busy)
            flushed = time_device(torch, fn, args.steps, args.warmup, flush)
            barrier(world)
            torch.cuda.synchronize()
        kernel_ms = sum(times) / len(times)
        step_ms = reduce_max(kernel_ms, world)
        flushed_ms = reduce_max(sum(flushed) / len(flushed), world)
        # e2e: the cache lives on the device (it is the model's KV cache); per step the host
        # sends q and the lengths and reads back O and LSE.
        hq = q.cpu().pin_memory()
        hlens = lens.cpu().pin_memory()
        ho = torch.empty(q.shape, dtype=torch.bfloat16, pin_memory=True)
        hl = torch.empty(q.shape[:-1], dtype=torch.float32, pin_memory=True)

        def e2e():
            dq = hq.to("cuda", non_blocking=True)
            dl = hlens.to("cuda", non_blocking=True)
            o, lse = student.attention_with_lse(dq, k, v, c["Tk"] - 1, None, dl)
            ho.copy_(o, non_blocking=True)
            hl.copy_(lse, non_blocking=True)
        e2e_ms = sum(time_device(torch, e2e, max(3, args.steps // 2), 2)) / max(3, args.steps // 2)
        e2e_ms = reduce_max(e2e_ms, world)
        achieved = nbytes / (kernel_ms * 1e-3) / 1e9
        tr = traffic.get("decode_split_kernel")
        results["decode"] = {
            "metric": "decode KV GB/s",
            "value": round(world * nbytes / (step_ms * 1e-3) / 1e9, 1),
            "unit": "GB/s",
            "ms_per_step": round(step_ms, 4),
            "config": {"workload": "cfg4 decode B=64 H=12 Tk=8192 D=64 bf16, kv_lens U[1024,8192] "
                                   f"seed {c['seed']}+rank, per rank",
                       "global_batch": c["B"] * world, "heads": c["H"], "kv_capacity": c["Tk"],
                       "sum_kv_lens_rank0": int(lens_np.sum()), "algorithmic_bytes": nbytes,
                       "parallelism": f"batch shards, {world} rank(s)",
                       "l2": "inputs larger than L2 (K/V read ~0.9 GB, 7x L2), no flush; a "
                             "spin kernel ahead of each step keeps host latency out"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"],
                         "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4),
                         "peak_kind": f"{peaks['source']} copy bandwidth", "traffic": tr,
                         "algorithmic_bytes": nbytes},
            "e2e": {"value": round(world * nbytes / (e2e_ms * 1e-3) / 1e9, 1), "unit": "GB/s",
                    "ms_per_step": round(e2e_ms, 4),
                    "h2d_bytes_per_step": hq.numel() * 2 + hlens.numel() * 4,
                    "d2h_bytes_per_step": ho.numel() * 2 + hl.numel() * 4},
            "gpu_launches": args.steps,
            "flushed": {"value": round(world * nbytes / (flushed_ms * 1e-3) / 1e9, 1),
                        "ms_per_step": round(flushed_ms, 4),
                        "l2": "256 MiB write between timed steps"},
            "clocks": clk.summary(),
        }

    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    if rank != 0:
        return
    head_key = "decode" if args.workload == "decode" else "prefill"
    other_key = "prefill" if head_key == "decode" else "decode"
    head = results[head_key]
    line = {
        "metric": head["metric"], "value": head["value"], "unit": head["unit"], "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": head["ms_per_step"],
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic N(0,1), seeded", "impl": "ours", "config": head["config"],
        "roofline": head["roofline"], "e2e": head["e2e"], "gpu_launches": head["gpu_launches"],
        "clocks": head["clocks"],
        "cpu_baseline": cpu_baseline(head_key, budget_s=args.cpu_budget) if world == 1 else None,
    }
    if "sdpa" in head:
        line["sdpa"] = head["sdpa"]
    line[other_key] = results[other_key]
    line["backward"] = results["backward"]
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- CPU side
def _cpu_workers():
    """Host threads for the CPU oracle: all cores available to this process, capped at 32 so
    the per-thread score matrices (~0.3 GB each at T=4096) stay well inside host memory."""
    n = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    return max(1, min(int(n or 1), 32))


def cpu_sample(workload, n_items, rank_seed=0):
    """Run the oracle port on `n_items` units of the workload in a thread pool (one unit per
    thread, BLAS limited to one thread each). Returns (seconds, algorithmic units done)."""
    from concurrent.futures import ThreadPoolExecutor

    from threadpoolctl import threadpool_limits

    from oracle import attention_oracle as oracle
    rng = np.random.default_rng(99 + rank_seed)
    if workload == "prefill":
        T = PREFILL_CFG["T"]
        items = [[oracle.round_bf16(rng.standard_normal((1, 1, T, 64), dtype=np.float32))
                  for _ in range(3)] for _ in range(n_items)]
        work = lambda it: oracle.reference_attention_bf16(*it, 0, return_lse=True)  # noqa: E731
        unit = oracle.prefill_flops(1, 1, T, T, 0)
    else:
        c = DECODE_CFG
        lens = decode_lengths(c, 0)
        items = []
        for i in range(n_items):
            L = int(lens[i % len(lens)])
            items.append(([oracle.round_bf16(rng.standard_normal((1, c["H"], 1, 64), dtype=np.float32))]
                          + [oracle.round_bf16(rng.standard_normal((1, c["H"], L, 64), dtype=np.float32))
                             for _ in range(2)], L))
        work = lambda it: oracle.reference_attention_bf16(*it[0], it[1] - 1, return_lse=True)  # noqa: E731
        unit = None
    with threadpool_limits(limits=1):
        t0 = time.perf_counter()
        with ThreadPoolExecutor(max_workers=_cpu_workers()) as pool:
            list(pool.map(work, items))
        dt = time.perf_counter() - t0
    if workload == "prefill":
        done = unit * n_items
    else:
        done = sum(oracle.decode_bytes(1, DECODE_CFG["H"], [it[1]]) for it in items)
    return dt, done


def cpu_baseline(workload, budget_s=20.0):
    cores = _cpu_workers()
    if workload == "prefill":
        dt, flops = cpu_sample("prefill", cores)
        value, unit = flops / dt / 1e12, "TFLOP/s"
        sample = (f"{cores} (batch, head) slices of cfg3 (Tq=Tk=4096, causal), one per thread, "
                  f"numpy oracle port, {dt:.1f} s")
    else:
        n = cores * 4
        dt, nbytes = cpu_sample("decode", n)
        value, unit = nbytes / dt / 1e9, "GB/s"
        sample = f"{n} sequences of cfg4 (12 heads, lengths from the cfg4 seed), numpy oracle port, {dt:.1f} s"
    return {"value": round(value, 5), "unit": unit, "cores": cores, "kind": "port", "sample": sample}


def run_reference(args):
    world, rank, _ = init_dist()
    if rank != 0:
        return
    workload = "decode" if args.workload == "decode" else "prefill"
    cores = _cpu_workers()
    times, done_total = [], 0
    for i in range(args.warmup + args.steps):
        n = cores if workload == "prefill" else cores * 4
        dt, done = cpu_sample(workload, n, rank_seed=i)
        if i >= args.warmup:
            times.append(dt)
            done_total += done
    total = sum(times)
    if workload == "prefill":
        value, unit, metric = done_total / total / 1e12, "TFLOP/s", "causal attn fwd TFLOP/s (prefill)"
        cfg = {"workload": "cfg3 causal prefill B=4 H=12 Tq=Tk=4096 D=64 bf16 N(0,1)",
               "sample_per_step": f"{cores} (batch, head) slices"}
    else:
        value, unit, metric = done_total / total / 1e9, "GB/s", "decode KV GB/s"
        cfg = {"workload": "cfg4 decode B=64 H=12 Tk=8192 D=64 bf16, kv_lens U[1024,8192]",
               "sample_per_step": f"{cores * 4} sequences"}
    line = {
        "metric": metric, "value": round(value, 5), "unit": unit, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 * total / len(times), 2),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic N(0,1), seeded", "impl": "reference", "config": cfg,
        "cpu_baseline": {"value": round(value, 5), "unit": unit, "cores": cores, "kind": "port",
                         "sample": f"{cfg['sample_per_step']} per step, numpy restatement of "
                                   "reference.attention (oracle/attention_oracle.py)"},
        "e2e": {"value": round(value, 5), "unit": unit, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


GEN_CFG = {"batch": 32, "prompt": 128, "new_tokens": 256, "seed": 1234}


def run_generation(args):
    """greedy generation with a random-init decoder shaped like the
    reference's configs/model_60m.json (8 layers, dim 768, 12 x 64 heads, SwiGLU 2048, vocab
    8192, tied, BF16 N(0, 0.02) weights), batch 32, prompt 128 ids uniform in [0, 8192) by seed,
    256 new tokens. Timed like the reference's model benchmark (benchmarks/model.py): host wall
    time around device synchronisations, one warm-up request, medians over ``--steps`` requests.
    Attention backends: student eager (the reference's call sequence, cache prefix views read in
    place), student graphed (one CUDA graph per decode step over the full-capacity cache with
    device-held kv_lens), torch SDPA and the reference specification. One GPU; under torchrun
    only rank 0 runs."""
    import statistics

    import torch
    import __graft_entry__
    __graft_entry__.import_package()
    from tiny_transformer_b200.generation import Decoder, DecoderConfig, request

    if int(os.environ.get("RANK", "0")) != 0:
        return
    torch.manual_seed(GEN_CFG["seed"])
    model = Decoder(DecoderConfig(), "student").to(device="cuda", dtype=torch.bfloat16).eval()
    g = torch.Generator(device="cuda").manual_seed(GEN_CFG["seed"])
    prompt = torch.randint(0, model.config.vocab_size, (GEN_CFG["batch"], GEN_CFG["prompt"]),
                           device="cuda", generator=g)
    repeats = max(1, min(args.steps, 5))
    results = {}
    for name, backend, graphed in (("student_graphed", "student", True),
                                   ("student", "student", False), ("sdpa", "sdpa", False),
                                   ("reference", "reference", False)):
        model.set_attention(backend)
        request(model, prompt, GEN_CFG["new_tokens"], graphed=graphed)  # warm-up
        trials = [request(model, prompt, GEN_CFG["new_tokens"], graphed=graphed)
                  for _ in range(repeats)]
        results[name] = {k: round(statistics.median(t[k] for t in trials), 4)
                         for k in ("ttft_ms", "tpot_ms", "request_ms",
                                   "output_tokens_per_second", "decode_tokens_per_second")}
    head = results["student_graphed"]
    line = {
        "metric": "decode_tokens_per_second", "value": head["decode_tokens_per_second"],
        "unit": "tokens/s", "n_gpus": 1, "steps": repeats, "warmup": 1,
        "ms_per_step": head["request_ms"], "higher_is_better": True, "scaling": "none",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic ids, random-init weights",
        "config": {"workload": "cfg5 greedy generation, model_60m shape, batch 32, prompt 128, "
                               "256 new tokens, attention=student (graphed decode)",
                   "kv_capacity": GEN_CFG["prompt"] + GEN_CFG["new_tokens"]},
        "backends": results,
    }
    print(json.dumps(line), flush=True)


def run_profile_case(which):
    """A few launches of one kernel at BASELINE size, for ncu captures (no timing, no CPU leg):
    two warm-up calls then one profiled call."""
    import torch
    import __graft_entry__
    __graft_entry__.import_package()
    from tiny_transformer_b200.operators._extension import load_attention_extension
    ext = load_attention_extension()
    with torch.no_grad():
        if which == "prefill":
            q, k, v = make_prefill(torch, 0)
            for _ in range(3):
                ext.attention_forward(q, k, v, 0)
        elif which == "backward":
            q, k, v = make_prefill(torch, 0)
            out, lse = ext.attention_forward(q, k, v, 0)
            dout = torch.randn_like(out)
            for _ in range(3):
                ext.attention_backward(q, k, v, dout, out, lse, 0)
        else:
            q, k, v, lens = make_decode(torch, 0)
            for _ in range(3):
                ext.attention_forward(q, k, v, DECODE_CFG["Tk"] - 1, None, lens)
    torch.cuda.synchronize()
    print(f"profile case {which} done")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", choices=("prefill", "decode", "generation"), default="prefill")
    ap.add_argument("--cpu-budget", type=float, default=20.0)
    ap.add_argument("--profile", choices=("prefill", "decode", "backward"), default=None,
                    help="run 3 launches of one kernel for an ncu capture and exit")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.profile:
        run_profile_case(args.profile)
        return
    if args.workload == "generation":
        run_generation(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
