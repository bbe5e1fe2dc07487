#!/usr/bin/env python
"""Benchmark of the B200 chunked linear cross-entropy hot path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--workload lce|ce|sls]

Default workload (``lce``): Llama-3-8B LM head, ``chunked_linear_cross_entropy``
forward + backward through the public API with H[8192, 4096] (RMS-normalised
N(0,1)), W[128256, 4096] ~ N(0, 0.02), bf16, 2% ignore_index, mean reduction.
With N GPUs (torchrun, one process per GPU) every rank runs its own 8192 rows
(data-parallel, weight replicated, weight gradient all-reduced over NCCL):
weak scaling, ``value`` = total tokens/s over all ranks.

One JSON line is printed by rank 0. Timing: W warm-up steps, then K steps
between barrier + synchronize, device time from CUDA events, max over ranks.
``--workload ce`` / ``sls`` time the standalone row kernels (GB/s).
``--impl reference`` times the reference's own PyTorch path on the host cores
(bf16 ``F.linear``, ``F.cross_entropy`` on fp32 logits, autograd backward:
oracle/torch_path.py) on contiguous row samples of the same workload; the
reference's fused kernels are CuTe-DSL and GPU-only, and its checkout is not
on the GPU box.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "linear-CE fwd+bwd tokens/s, Llama-3-8B head; % bf16 TC peak @1/2/4/8 GPU"
# DRAM bytes (read + write) per launch from one ncu capture of each kernel class
# at the bench workload (one-pass ncu capture of each GEMM class); None if not captured.
TRAFFIC_BYTES_PER_LAUNCH: dict = {
    # Llama-3-8B head, one chunk, q-store pipeline: DRAM read + write per
    # launch (profiles/tc_gemm_cfg3_traffic.md)
    "gemm_logits_ce": 9.471e9 + 2.116e9,
    "gemm_dw": 15.047e9 + 1.035e9,
    "gemm_dh": 17.082e9 + 0.124e9,
}
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def load_peaks() -> tuple[dict, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text()), "measured"
    return dict(PEAKS_FALLBACK), "fallback"


# --------------------------------------------------------------------------- dist

def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    allv = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(allv, t)
    PER_RANK.append([round(float(v.item()), 4) for v in allv])
    return max(float(v.item()) for v in allv)


PER_RANK: list = []  # every max_over_ranks call's per-rank values, for the JSON line


# --------------------------------------------------------------------------- clocks

class ClockSampler:
    """nvidia-smi clocks/throttle sampling during the timed region."""

    FIELDS = "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"

    def __init__(self, device_index: int):
        self.idx = device_index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL,
            )
        except Exception:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self) -> dict:
        out = {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        if not self.path or not os.path.exists(self.path):
            return out
        rows = [r.split(",") for r in Path(self.path).read_text().strip().splitlines() if r.strip()]
        os.unlink(self.path)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            r = [c.strip() for c in r]
            if len(r) < 9:
                continue
            try:
                sm.append(float(r[1]))
                mx.append(float(r[2]))
            except ValueError:
                continue
            for n, v in zip(names, r[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if sm:
            out.update(sm_mhz=statistics.median(sm), sm_max_mhz=max(mx), reasons=sorted(reasons), samples=len(sm))
        return out


# --------------------------------------------------------------------------- workloads

def make_lce_inputs(N, D, V, seed, device, w_std=0.02, ignore_frac=0.02):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    H = torch.randn(N, D, device=device, generator=g)
    H = H * torch.rsqrt(H.square().mean(-1, keepdim=True) + 1e-6)
    W = (torch.randn(V, D, device=device, generator=g) * w_std).to(torch.bfloat16)
    t = torch.randint(0, V, (N,), device=device, generator=g)
    ign = torch.rand(N, device=device, generator=g) < ignore_frac
    t[ign] = -100
    return H.to(torch.bfloat16), W, t


def time_steps(step, steps, warmup, world):
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        step()
    end.record()
    torch.cuda.synchronize()
    barrier(world)
    ms = start.elapsed_time(end) / steps
    return max_over_ranks(ms, world)


def cpu_threads() -> int:
    try:
        from threadpoolctl import threadpool_info

        n = [i.get("num_threads", 1) for i in threadpool_info() if i.get("user_api") == "blas"]
        if n:
            return int(max(n))
    except Exception:
        pass
    return os.cpu_count() or 1


def cpu_baseline_lce(N, D, V, rows=512, repeats=3):
    """The reference's own torch path (bf16 F.linear, F.cross_entropy on fp32
    logits, autograd backward) on one contiguous row sample of the workload,
    on all host threads (oracle/torch_path.py)."""
    from oracle.torch_path import time_linear_ce

    r = time_linear_ce(N, D, V, rows=rows, repeats=repeats, threads=os.cpu_count() or 1)
    r["kind"] = "port"
    r["port_of"] = "reference torch path (src/tests/nn/functional/chunked_linear_loss_test.py:18-42)"
    return r


def bench_lce(args, rank, world, local):
    from greyhound_b200 import _lib
    from greyhound_b200.nn.functional import chunked_linear_cross_entropy

    N, D, V = args.rows or 8192, args.hidden or 4096, args.vocab or 128256
    dev = torch.device("cuda", local)
    # the standalone row kernels at their configs (cfg2, cfg4), measured first,
    # on a GPU not yet heated by the GEMMs
    rows_block = row_kernel_block(local) if world == 1 and not args.no_extras else None
    H, W, t = make_lce_inputs(N, D, V, 2 + rank, dev)
    H.requires_grad_(True)
    W.requires_grad_(True)
    if world > 1:
        from greyhound_b200.distributed import row_sharded_linear_cross_entropy as fn
    else:
        fn = chunked_linear_cross_entropy

    def step():
        H.grad = None
        W.grad = None
        loss = fn(H, W, t)
        loss.backward()

    # device-resident timing; the library brackets its launches with CUDA
    # events per kernel class (on the launching stream) for the roofline
    c0 = _lib.launch_count()
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    _lib.profile_read(reset=True)
    _lib.profile_enable(True)
    with ClockSampler(local) as clk:
        ms = time_steps(step, args.steps, 0, world)
    _lib.profile_enable(False)
    prof = _lib.profile_read(reset=True)
    launches = (_lib.launch_count() - c0) // (args.steps + args.warmup)
    clocks = clk.summary()
    # peak device memory of one step, measured as the reference bench does
    # (src/benchmarks/chunked_linear_cross_entropy_bench.py:182-190)
    torch.cuda.synchronize()
    torch.cuda.reset_peak_memory_stats(dev)
    step()
    torch.cuda.synchronize()
    peak_mem_mb = torch.cuda.max_memory_allocated(dev) / 2**20

    # end-to-end: each step's H/targets copied from pinned host memory and its
    # loss read back. The copy of step k+1's inputs is issued on a copy stream
    # while step k computes (double-buffered, as a training input pipeline
    # does); the first timed step copies its own inputs inside the timed region.
    H_host = H.detach().cpu().pin_memory()
    t_host = t.cpu().pin_memory()
    loss_host = torch.empty((), dtype=torch.float32).pin_memory()
    bufs = [(torch.empty_like(H.detach()), torch.empty_like(t)) for _ in range(2)]
    copy_stream = torch.cuda.Stream(device=dev)
    state = {"k": 0, "ready": None, "done": [None, None]}

    def issue(k):
        Hb, tb = bufs[k % 2]
        prev = state["done"][k % 2]
        with torch.cuda.stream(copy_stream):
            if prev is not None:
                copy_stream.wait_event(prev)  # the step that last used this buffer is finished
            Hb.copy_(H_host, non_blocking=True)
            tb.copy_(t_host, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(copy_stream)
        return ev

    def e2e_step():
        k = state["k"]
        ev = state["ready"] if state["ready"] is not None else issue(k)
        torch.cuda.current_stream().wait_event(ev)
        state["ready"] = issue(k + 1)
        Hb, tb = bufs[k % 2]
        Hin = Hb.detach().requires_grad_(True)
        W.grad = None
        loss = fn(Hin, W, tb)
        loss.backward()
        loss_host.copy_(loss.detach(), non_blocking=True)
        done = torch.cuda.Event()
        done.record()
        state["done"][k % 2] = done
        state["k"] = k + 1

    for _ in range(args.warmup):
        e2e_step()
    torch.cuda.synchronize()
    state["ready"] = None  # the first timed step copies its own inputs
    ms_e2e = time_steps(e2e_step, args.steps, 0, world)
    # the last prefetch belongs to a step outside the timed region
    torch.cuda.synchronize()

    peaks, peak_src = load_peaks()
    flops = 6.0 * N * D * V
    tflops = flops / (ms * 1e-3) / 1e12
    value = N * world / (ms * 1e-3)
    # per-kernel-class device time over the timed steps (CUDA events)
    gemm_flops = 2.0 * N * D * V  # each of the three GEMMs per step (one chunk at this size)
    kernels = {}
    for cls, (tot_ms, cnt) in prof.items():
        if cnt:
            per = tot_ms / cnt
            k = {"launches_per_step": cnt / args.steps, "ms_per_launch": per,
                 "share_of_step": tot_ms / (ms * args.steps)}
            if cls.startswith("gemm_") and cls != "gemm_other":
                k["tflops"] = gemm_flops / (per * 1e-3) / 1e12
            if cls == "glue":  # the small kernels between the GEMMs (q fix-up, target column, alpha * H)
                k["note"] = "q fix-up, target column, alpha*H (or the logits -> dlogits pass when q mode is off)"
            kernels[cls] = k
    gemms = [c for c in kernels if c.startswith("gemm_") and c != "gemm_other"]
    dom = max(gemms, key=lambda c: kernels[c]["share_of_step"], default=None)
    timed_s = ms * args.steps * 1e-3
    if dom is not None:
        ach = kernels[dom]["tflops"]
        roofline = roofline_tensor(ach, peaks, peak_src, timed_s)
        roofline.update(kernel=dom, algorithmic_flops_per_launch=gemm_flops,
                        traffic=TRAFFIC_BYTES_PER_LAUNCH.get(dom))
    else:
        roofline = None
    line = {
        "metric": METRIC,
        "value": value,
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded randn of the workload's shapes; no dataset)",
        "config": {
            "workload": "Llama-3-8B LM head chunked_linear_cross_entropy fwd+bwd (BASELINE configs[2])"
            if (N, D, V) == (8192, 4096, 128256) else f"profiling case N={N} D={D} V={V}",
            "N_per_rank": N, "D": D, "V": V, "global_tokens": N * world,
            "reduction": "mean", "ignore_frac": 0.02,
            "parallelism": f"dp{world} (row-sharded, dW all-reduce)" if world > 1 else "single GPU",
            "l2": "inputs larger than L2 (W = 1.05 GB bf16)",
        },
        "tflops_per_gpu": tflops,
        "frac_of_bf16_peak": tflops / peaks["bf16_tflops"],
        "roofline": roofline,
        "kernels": kernels,
        "e2e": {
            "value": N * world / (ms_e2e * 1e-3),
            "unit": "tokens/s",
            "ms_per_step": ms_e2e,
            "h2d_bytes_per_step": H.numel() * 2 + t.numel() * 8,
            "d2h_bytes_per_step": 4,
            "input_pipeline": "pinned host -> device copy of every step's inputs, issued one step ahead on a copy stream",
        },
        "gpu_launches": launches * args.steps,
        "gpu_launches_per_step": launches,
        "clocks": clocks,
        "peak_mem_mb": peak_mem_mb,
    }
    if world > 1:
        line["ms_per_rank"] = {"device": PER_RANK[0], "e2e": PER_RANK[-1]}
        from greyhound_b200 import distributed as _dd

        if _dd._DP_TIMING:
            line["dp_phases_ms"] = _dd.dp_phase_summary()
    del H, W, bufs
    torch.cuda.empty_cache()
    if rows_block is not None:
        line["row_kernels"] = rows_block
    if world == 1 and not args.no_extras and (N, D, V) == (8192, 4096, 128256):
        # same-box comparators, so the driver's run measures them too
        line["comparators"] = comparators(args)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_lce(N, D, V)
    return line


def roofline_tensor(ach: float, peaks: dict, src: str, timed_s: float) -> dict:
    """Tensor-core roofline of a kernel timed over ``timed_s`` seconds: the
    burst cuBLAS peak for a short timed region (the clocks stay near maximum),
    the sustained one (measured over 4 s at the 1 kW cap) for >= 4 s."""
    sustained = timed_s >= 4.0 and "bf16_tflops_sustained" in peaks
    peak = peaks["bf16_tflops_sustained"] if sustained else peaks["bf16_tflops"]
    r = {"bound": "tensor", "achieved": ach, "peak": peak, "unit": "TFLOP/s", "frac": ach / peak,
         "peak_source": f"{src} {'sustained' if sustained else 'burst'} cuBLAS bf16 "
                        f"(timed region {timed_s:.2f} s)",
         "frac_of_spec_2250": ach / 2250.0}
    if "bf16_tflops_sustained" in peaks:
        r["frac_of_sustained_peak"] = ach / peaks["bf16_tflops_sustained"]
    return r


def _row_case(which: str, rows: int, V: int, dev, steps: int = 30, warmup: int = 10) -> dict:
    from greyhound_b200.kernels.cross_entropy import cross_entropy_with_grad
    from greyhound_b200.kernels.logprobs import (
        selective_log_softmax_backward_kernel,
        selective_log_softmax_with_lse,
    )

    g = torch.Generator(device=dev)
    g.manual_seed(1 if which == "ce" else 3)
    if which == "ce":
        x = (torch.randn(rows, V, device=dev, generator=g) * 2).to(torch.bfloat16)
        t = torch.randint(0, V, (rows,), device=dev, generator=g)
        out = torch.empty_like(x)
        step = lambda: cross_entropy_with_grad(x, t, 0.0, -100, out, mean_reduction=True)  # noqa: E731
        nbytes = 2 * rows * V * 2 + rows * 8
    else:
        x = (torch.randn(rows, V, device=dev, generator=g) * 3).to(torch.bfloat16)
        t = torch.randint(0, V, (rows,), device=dev, generator=g)
        if which == "sls":
            step = lambda: selective_log_softmax_with_lse(x, t, out_dtype=torch.float32)  # noqa: E731
            nbytes = rows * V * 2 + rows * 8 + rows * 4
        else:
            _, lse = selective_log_softmax_with_lse(x, t, out_dtype=torch.float32)
            go = torch.randn(rows, device=dev, generator=g)
            step = lambda: selective_log_softmax_backward_kernel(x, t, lse, go)  # noqa: E731
            nbytes = 2 * rows * V * 2 + rows * (8 + 4 + 4)
    ms = time_steps(step, steps, warmup, 1)
    del x
    torch.cuda.empty_cache()
    return {"rows": rows, "V": V, "ms": ms, "gbs": nbytes / (ms * 1e-3) / 1e9, "algorithmic_bytes": nbytes}


def row_kernel_block(local: int) -> dict:
    """CE fwd+grad on [4096, 128256] and [16, 128256] (cfg2), selective
    log-softmax forward and backward on [65536, 151936] (cfg4), bf16; GB/s of
    algorithmic bytes and the fraction of the measured HBM copy bandwidth.
    The big cases' inputs exceed L2; the 16-row case is L2-resident and
    latency-bound, reported for completeness."""
    dev = torch.device("cuda", local)
    peaks, src = load_peaks()
    out = {"peak_gbs": peaks["hbm_gbs"], "peak_source": f"{src} HBM copy"}
    for name, which, rows, V in (("ce_cfg2", "ce", 4096, 128256), ("ce_cfg2_16rows", "ce", 16, 128256),
                                 ("sls_fwd_cfg4", "sls", 65536, 151936), ("sls_bwd_cfg4", "sls_bwd", 65536, 151936)):
        r = _row_case(which, rows, V, dev)
        r["frac"] = r["gbs"] / peaks["hbm_gbs"]
        out[name] = r
    return out


def comparators(args) -> dict:
    """Same-box comparators of the cfg3 step, each in a child process with a
    time limit: the reference's own GPU implementation
    (``greyhound.nn.functional.chunked_linear_cross_entropy``, installed
    unmodified under baseline/_ref), and the reference bench's torch-eager
    and torch-compile providers (src/benchmarks/third_party/torch.py)."""
    res = {}
    for prov in ("greyhound_reference", "torch_eager", "torch_compile"):
        cmd = [sys.executable, str(ROOT / "bench.py"), "--comparator-child", prov,
               "--steps", "10", "--warmup", "3"]
        try:
            p = subprocess.run(cmd, capture_output=True, text=True, timeout=420)
            last = [ln for ln in p.stdout.splitlines() if ln.startswith("{")]
            res[prov] = json.loads(last[-1]) if last else {
                "unavailable": (p.stderr.strip().splitlines() or ["no output"])[-1][:300]}
        except subprocess.TimeoutExpired:
            res[prov] = {"unavailable": "timed out after 420 s"}
    return res


def comparator_child(prov: str, steps: int, warmup: int) -> dict:
    N, D, V = 8192, 4096, 128256
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    H, W, t = make_lce_inputs(N, D, V, 2, dev)
    H.requires_grad_(True)
    W.requires_grad_(True)
    if prov == "greyhound_reference":
        ref = ROOT / "baseline" / "_ref"
        if not (ref / "greyhound").exists():
            return {"unavailable": "reference not installed under baseline/_ref"}
        sys.path.insert(0, str(ref))
        from greyhound.nn.functional import chunked_linear_cross_entropy as fn
    else:
        import torch.nn.functional as F

        def fn(inputs, weight, target):  # src/benchmarks/third_party/torch.py:9-30
            logits = inputs @ weight.T
            return F.cross_entropy(logits.float(), target, ignore_index=-100, reduction="mean")

        if prov == "torch_compile":
            fn = torch.compile(fn)

    def step():
        H.grad = None
        W.grad = None
        fn(H, W, t).backward()

    ms = time_steps(step, steps, warmup, 1)
    torch.cuda.reset_peak_memory_stats(dev)
    step()
    torch.cuda.synchronize()
    return {"ms_per_step": ms, "tokens_per_s": N / (ms * 1e-3), "tflops": 6.0 * N * D * V / (ms * 1e-3) / 1e12,
            "peak_mem_mb": torch.cuda.max_memory_allocated(dev) / 2**20, "steps": steps, "warmup": warmup}


def bench_lce70b(args, rank, world, local):
    """Llama-3-70B-scale head workload: H[65536, 8192], W[128256, 8192]
    ~N(0, 0.015), 2% ignore, mean. ``--parallel rows``: the 65536 rows split over
    the ranks, W replicated, dW all-reduced; ``--parallel vocab``: W split by
    vocabulary rows, H replicated, per-row statistics all-gathered and the
    partial dH all-reduced. Total work fixed: strong scaling."""
    from greyhound_b200 import _lib
    from greyhound_b200.distributed import (
        row_sharded_linear_cross_entropy,
        shard_range,
        vocab_sharded_linear_cross_entropy,
    )
    from greyhound_b200.nn.functional import chunked_linear_cross_entropy

    N, D, V = args.rows or 65536, args.hidden or 8192, args.vocab or 128256
    dev = torch.device("cuda", local)
    g = torch.Generator(device=dev)
    if args.parallel == "vocab" and world > 1:
        g.manual_seed(4)  # identical H / targets on every rank
        H = torch.randn(N, D, device=dev, generator=g).to(torch.bfloat16)
        t = torch.randint(0, V, (N,), device=dev, generator=g)
        t[torch.rand(N, device=dev, generator=g) < 0.02] = -100
        vs, ve = shard_range(V, rank, world)
        g.manual_seed(1000 + rank)
        W = (torch.randn(ve - vs, D, device=dev, generator=g) * 0.015).to(torch.bfloat16)
        fn = lambda h, w, tt: vocab_sharded_linear_cross_entropy(h, w, tt, vs)  # noqa: E731
        par = f"vocab-parallel x{world} (stats all-gather + dH all-reduce)"
    else:
        rs, re_ = shard_range(N, rank, world)
        g.manual_seed(4 + rank)
        H = torch.randn(re_ - rs, D, device=dev, generator=g).to(torch.bfloat16)
        t = torch.randint(0, V, (re_ - rs,), device=dev, generator=g)
        t[torch.rand(re_ - rs, device=dev, generator=g) < 0.02] = -100
        g.manual_seed(1000)
        W = (torch.randn(V, D, device=dev, generator=g) * 0.015).to(torch.bfloat16)
        fn = row_sharded_linear_cross_entropy if world > 1 else chunked_linear_cross_entropy
        par = f"row-sharded x{world} (dW all-reduce)" if world > 1 else "single GPU"
    H.requires_grad_(True)
    W.requires_grad_(True)

    def step():
        H.grad = None
        W.grad = None
        fn(H, W, t).backward()

    c0 = _lib.launch_count()
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    _lib.profile_read(reset=True)
    _lib.profile_enable(True)
    with ClockSampler(local) as clk:
        ms = time_steps(step, args.steps, 0, world)
    _lib.profile_enable(False)
    prof = _lib.profile_read(reset=True)
    launches = (_lib.launch_count() - c0) // (args.steps + args.warmup)
    peaks, src = load_peaks()
    tflops_gpu = 6.0 * N * D * V / world / (ms * 1e-3) / 1e12
    kernels = {c: {"launches_per_step": n / args.steps, "ms_per_step": tot / args.steps}
               for c, (tot, n) in prof.items() if n}
    return {
        "metric": "linear-CE fwd+bwd tokens/s, Llama-3-70B-scale head", "value": N / (ms * 1e-3),
        "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded randn of the workload's shapes)",
        "config": {"workload": "Llama-3-70B-scale head chunked_linear_cross_entropy fwd+bwd (BASELINE configs[4])",
                   "N": N, "D": D, "V": V, "parallelism": par, "l2": "inputs larger than L2"},
        "tflops_per_gpu": tflops_gpu,
        "roofline": dict(roofline_tensor(tflops_gpu, peaks, src, ms * args.steps * 1e-3),
                         kernel="whole step (6*N*D*V / GPUs)", traffic=None),
        "kernels": kernels, "gpu_launches": launches * args.steps, "clocks": clk.summary(),
    }


def bench_reference(args, rank, world):
    """The reference's own torch path (oracle/torch_path.py) on the host cores:
    each step is one contiguous ``--ref-rows``-row sample of the workload
    (forward, backward, one dW), tokens/s = sample rows / sample time. Rank 0
    alone runs it."""
    if rank != 0:
        return None
    from oracle.torch_path import time_linear_ce

    N, D, V = args.rows or 8192, args.hidden or 4096, args.vocab or 128256
    rows = min(args.ref_rows, N)
    r = time_linear_ce(N, D, V, rows=rows, repeats=args.warmup + args.steps, threads=os.cpu_count() or 1)
    v = r["value"]
    cb = {"value": v, "unit": "tokens/s", "cores": r["cores"], "kind": "port",
          "port_of": "reference torch path (src/tests/nn/functional/chunked_linear_loss_test.py:18-42)",
          "sample": r["sample"]}
    return {
        "impl": "reference",
        "metric": METRIC,
        "value": v,
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": 1e3 * N / v,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16 GEMMs, fp32 CE (torch CPU)",
        "data": "synthetic",
        "config": {"workload": "Llama-3-8B LM head chunked_linear_cross_entropy fwd+bwd (BASELINE configs[2])"
                   if (N, D, V) == (8192, 4096, 128256) else f"profiling case N={N} D={D} V={V}",
                   "N_per_rank": N, "D": D, "V": V, "global_tokens": N * world,
                   "reduction": "mean", "ignore_frac": 0.02, "parallelism": "host CPU",
                   "l2": "n/a (host)"},
        "cpu_baseline": cb,
        "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def bench_rows(args, rank, world, local, which):
    """Standalone row kernels: CE+grad on [4096, 128256] (cfg2) or SLS fwd on
    [65536, 151936] (cfg4), bf16. GB/s with the reference bench formulas."""
    from greyhound_b200 import _lib
    from greyhound_b200.kernels.cross_entropy import cross_entropy_with_grad
    from greyhound_b200.kernels.logprobs import selective_log_softmax_with_lse

    dev = torch.device("cuda", local)
    g = torch.Generator(device=dev)
    g.manual_seed(1 + rank)
    if which == "ce":
        rows, V = args.rows or 4096, args.vocab or 128256
        x = (torch.randn(rows, V, device=dev, generator=g) * 2).to(torch.bfloat16)
        t = torch.randint(0, V, (rows,), device=dev, generator=g)
        out = torch.empty_like(x)
        step = lambda: cross_entropy_with_grad(x, t, 0.0, -100, out, mean_reduction=True)  # noqa: E731
        nbytes = 2 * rows * V * 2 + rows * 8
        metric = f"cross_entropy fwd+grad GB/s [{rows},{V}] bf16"
    elif which == "sls":
        rows, V = args.rows or 65536, args.vocab or 151936
        x = (torch.randn(rows, V, device=dev, generator=g) * 3).to(torch.bfloat16)
        t = torch.randint(0, V, (rows,), device=dev, generator=g)
        step = lambda: selective_log_softmax_with_lse(x, t, out_dtype=torch.float32)  # noqa: E731
        nbytes = rows * V * 2 + rows * 8 + rows * 4
        metric = f"selective_log_softmax fwd GB/s [{rows},{V}] bf16"
    else:  # sls_bwd: grad_logits = g * (onehot - softmax), from the saved lse
        from greyhound_b200.kernels.logprobs import selective_log_softmax_backward_kernel

        rows, V = args.rows or 65536, args.vocab or 151936
        x = (torch.randn(rows, V, device=dev, generator=g) * 3).to(torch.bfloat16)
        t = torch.randint(0, V, (rows,), device=dev, generator=g)
        _, lse = selective_log_softmax_with_lse(x, t, out_dtype=torch.float32)
        go = torch.randn(rows, device=dev, generator=g)
        step = lambda: selective_log_softmax_backward_kernel(x, t, lse, go)  # noqa: E731
        nbytes = 2 * rows * V * 2 + rows * (8 + 4 + 4)
        metric = f"selective_log_softmax bwd GB/s [{rows},{V}] bf16"
    c0 = _lib.launch_count()
    with ClockSampler(local) as clk:
        ms = time_steps(step, args.steps, args.warmup, world)
    launches = (_lib.launch_count() - c0) // (args.steps + args.warmup)
    gbs = nbytes / (ms * 1e-3) / 1e9
    peaks, src = load_peaks()
    return {
        "metric": metric, "value": gbs * world, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": which, "rows": rows, "V": V, "l2": "inputs larger than L2"},
        "roofline": {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": gbs / peaks["hbm_gbs"], "peak_source": src, "traffic": None},
        "gpu_launches": launches * args.steps, "clocks": clk.summary(),
    }


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--workload", choices=["lce", "lce70b", "ce", "sls", "sls_bwd"], default="lce")
    ap.add_argument("--parallel", choices=["rows", "vocab"], default="rows", help="lce70b sharding mode")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true", help="skip the row-kernel block and the comparators")
    ap.add_argument("--comparator-child", default="", help=argparse.SUPPRESS)
    ap.add_argument("--ref-rows", type=int, default=512, help="rows per sample of the reference CPU arm")
    # shape overrides, only for small profiler captures (the default is the workload)
    ap.add_argument("--rows", type=int, default=0)
    ap.add_argument("--hidden", type=int, default=0)
    ap.add_argument("--vocab", type=int, default=0)
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.comparator_child:
        print(json.dumps(comparator_child(args.comparator_child, args.steps, args.warmup)), flush=True)
        return 0
    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        world = int(os.environ.get("WORLD_SIZE", "1"))
        line = bench_reference(args, rank, world)
        if line is not None:
            print(json.dumps(line), flush=True)
        return 0
    rank, world, local = dist_setup(args.gpus)
    if args.workload == "lce":
        line = bench_lce(args, rank, world, local)
    elif args.workload == "lce70b":
        line = bench_lce70b(args, rank, world, local)
    else:
        line = bench_rows(args, rank, world, local, args.workload)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
