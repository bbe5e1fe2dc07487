"""Benchmark timer.

Keeps the import path and signature of the reference's ``do_bench``
(src/greyhound/kernels/tuning_utils.py:6-24) but times with CUDA events on the
current stream instead of Triton: warm-up for ``warmup`` ms, then repeat for
about ``rep`` ms, flushing L2 between iterations by writing a 256 MB buffer
(larger than the B200's 126 MB L2).
"""

from __future__ import annotations

from typing import Callable

import torch


def do_bench(
    fn: Callable,
    warmup: int = 250,
    rep: int = 500,
    grad_to_none: list[torch.Tensor] | bool | None = None,
    quantiles: list[float] | None = None,
    return_mode: str = "mean",
) -> tuple | float:
    """Time ``fn`` in milliseconds; returns quantiles if given, else ``return_mode``."""
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device="cuda")
    fn()
    torch.cuda.synchronize()
    # estimate
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(5):
        flush.zero_()
        fn()
    end.record()
    torch.cuda.synchronize()
    est = max(start.elapsed_time(end) / 5, 1e-3)
    n_warm = max(1, int(warmup / est))
    n_rep = max(1, int(rep / est))
    for _ in range(n_warm):
        fn()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(n_rep)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(n_rep)]
    for i in range(n_rep):
        if isinstance(grad_to_none, list):
            for t in grad_to_none:
                t.grad = None
        flush.zero_()
        starts[i].record()
        fn()
        ends[i].record()
    torch.cuda.synchronize()
    times = torch.tensor([s.elapsed_time(e) for s, e in zip(starts, ends)], dtype=torch.float64)
    if quantiles is not None:
        q = torch.quantile(times, torch.tensor(quantiles, dtype=torch.float64)).tolist()
        return tuple(q) if len(q) > 1 else q[0]
    return float(getattr(torch, return_mode)(times).item())
