"""do_bench keeps the reference timer's interface
(src/greyhound/kernels/tuning_utils.py:6-24, Triton's do_bench conventions)
and agrees with a plain CUDA-event loop."""

import pytest
import torch

from greyhound_b200.kernels.tuning_utils import do_bench
from greyhound_b200.testing import requires_gpu


def _workload():
    a = torch.randn(4096, 4096, device="cuda", dtype=torch.bfloat16)
    return lambda: a @ a


@requires_gpu
def test_quantiles_are_ordered_and_match_an_event_loop():
    fn = _workload()
    q = do_bench(fn, warmup=20, rep=100, quantiles=[0.2, 0.5, 0.8])
    assert isinstance(q, list) and len(q) == 3
    assert 0 < q[0] <= q[1] <= q[2]
    # plain loop of CUDA events on the current stream, L2 flushed before each call
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device="cuda")
    times = []
    for _ in range(30):
        flush.zero_()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        times.append(s.elapsed_time(e))
    times.sort()
    assert abs(q[1] - times[15]) <= 0.25 * times[15]


@requires_gpu
def test_return_modes_and_single_quantile():
    fn = _workload()
    assert isinstance(do_bench(fn, warmup=5, rep=20, quantiles=[0.5]), float)
    allt = do_bench(fn, warmup=5, rep=20, return_mode="all")
    assert isinstance(allt, list) and len(allt) >= 1
    lo = do_bench(fn, warmup=5, rep=20, return_mode="min")
    hi = do_bench(fn, warmup=5, rep=20, return_mode="max")
    assert 0 < lo <= hi
    with pytest.raises(ValueError):
        do_bench(fn, return_mode="p99")


@requires_gpu
def test_grad_to_none_resets_gradients_before_each_call():
    x = torch.randn(1024, 1024, device="cuda", requires_grad=True)
    seen = []

    def fn():
        seen.append(x.grad is None)
        (x * 2).sum().backward()

    do_bench(fn, warmup=1, rep=5, grad_to_none=[x])
    n_timed = sum(1 for s in seen[-3:] if s)
    assert n_timed == 3  # every timed call started without an accumulated gradient
    with pytest.raises(TypeError):
        do_bench(fn, grad_to_none=True)
