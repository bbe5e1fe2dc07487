"""Device-side problems are reported to Python without a host sync and
without a GPU fault.

Kernels record a label outside [0, V) or a GEMM pipeline wait that ran out in
the workspace status word; every library call ends by OR-ing that word into a
per-device slot of pinned host memory, and the next Python-level call on the
device (or the autograd backward) raises: ValueError for a bad label (the
reference's kernels raise ValueError for bad inputs,
src/greyhound/kernels/cross_entropy.py:173-184), RuntimeError for a timeout.
The timeout is produced by the library's bounded-wait self-test (a GEMM whose
loads never arrive, 50 ms limit), nothing that can fault or hang the GPU."""

import pytest
import torch

from greyhound_b200 import _lib
from greyhound_b200.nn.functional import chunked_linear_cross_entropy, cross_entropy
from greyhound_b200.testing import requires_gpu


@requires_gpu
def test_pipeline_timeout_raises_at_the_next_call():
    lib = _lib.load()
    scratch = torch.zeros(128 * 1024, dtype=torch.uint8, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    st = lib.gh_gemm_selftest_stall(scratch.data_ptr(), scratch.numel(), status.data_ptr(), 50,
                                    torch.cuda.current_stream().cuda_stream)
    _lib.check(st, "selftest")
    torch.cuda.synchronize()
    x = torch.randn(8, 1000, device="cuda", dtype=torch.bfloat16)
    t = torch.randint(0, 1000, (8,), device="cuda")
    with pytest.raises(RuntimeError, match="timed out"):
        cross_entropy(x, t)
    # reported once; the context and the library keep working
    assert torch.isfinite(cross_entropy(x, t))


@requires_gpu
def test_bad_label_raises_at_the_next_call():
    x = torch.randn(4, 100, device="cuda", dtype=torch.bfloat16)
    loss = cross_entropy(x, torch.tensor([1, 200, -100, 3], device="cuda"))
    assert torch.isfinite(loss)  # the bad row counts as ignored, nothing faults
    torch.cuda.synchronize()
    with pytest.raises(ValueError, match="outside"):
        cross_entropy(x, torch.tensor([1, 2, -100, 3], device="cuda"))
    assert torch.isfinite(cross_entropy(x, torch.tensor([1, 2, -100, 3], device="cuda")))


@requires_gpu
def test_bad_target_of_linear_ce_raises_in_backward():
    g = torch.Generator(device="cuda").manual_seed(0)
    H = torch.randn(64, 128, device="cuda", generator=g).bfloat16().requires_grad_(True)
    W = (torch.randn(1000, 128, device="cuda", generator=g) * 0.05).bfloat16().requires_grad_(True)
    t = torch.randint(0, 1000, (64,), device="cuda", generator=g)
    t[5] = 1007
    loss = chunked_linear_cross_entropy(H, W, t)
    torch.cuda.synchronize()
    with pytest.raises(ValueError, match="outside"):
        loss.backward()


@requires_gpu
def test_clean_calls_leave_no_error_bits():
    x = torch.randn(64, 4096, device="cuda", dtype=torch.bfloat16)
    t = torch.randint(0, 4096, (64,), device="cuda")
    t[::7] = -100
    for _ in range(3):
        cross_entropy(x, t)
    torch.cuda.synchronize()
    assert _lib.take_device_errors(0) == 0
