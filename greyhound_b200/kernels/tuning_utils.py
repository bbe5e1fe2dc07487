"""Benchmark timer.

Keeps the import path, signature and return conventions of the reference's
``do_bench`` (src/greyhound/kernels/tuning_utils.py:6-24, which forwards to
``triton.testing.do_bench``) but times with CUDA events on the current stream
instead of Triton: about ``warmup`` ms of warm-up calls, then about ``rep`` ms
of timed calls, each preceded by a write of a 256 MB buffer (larger than the
B200's 126 MB L2) so that no call starts with a warm L2.

Return value, as Triton's: the ``quantiles`` of the per-call times in ms
(a list, or a float for a single quantile) when given, else the statistic
named by ``return_mode``: "min", "max", "mean", "median" or "all" (the list
of per-call times).
"""

from __future__ import annotations

import statistics
from typing import Callable, Iterable

import torch

_MODES = ("min", "max", "mean", "median", "all")


def do_bench(
    fn: Callable,
    warmup: int = 250,
    rep: int = 500,
    grad_to_none: Iterable[torch.Tensor] | None = None,
    quantiles: list[float] | None = None,
    return_mode: str = "mean",
) -> list[float] | float:
    """Time ``fn`` in milliseconds (see the module docstring).

    ``grad_to_none``: tensors whose ``.grad`` is reset to None before every
    timed call, so gradient accumulation is not timed."""
    if return_mode not in _MODES:
        raise ValueError(f"return_mode must be one of {_MODES}, got {return_mode!r}")
    if grad_to_none is not None and not isinstance(grad_to_none, (list, tuple)):
        raise TypeError("grad_to_none must be a list or tuple of tensors")
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device="cuda")
    fn()
    torch.cuda.synchronize()
    # estimate the time of one call (flush included) from 5 calls
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
        if grad_to_none is not None:
            for t in grad_to_none:
                t.grad = None
        flush.zero_()
        starts[i].record()
        fn()
        ends[i].record()
    torch.cuda.synchronize()
    times = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    if quantiles is not None:
        q = torch.quantile(torch.tensor(times, dtype=torch.float64),
                           torch.tensor(quantiles, dtype=torch.float64)).tolist()
        return q[0] if len(q) == 1 else q
    if return_mode == "all":
        return times
    return float({"min": min, "max": max, "mean": statistics.mean, "median": statistics.median}[return_mode](times))
