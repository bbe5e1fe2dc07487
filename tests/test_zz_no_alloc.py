"""The allocation-free cross-entropy entry point, gh_ce_fwd_grad_noalloc.

It exists for callers that cannot allocate device memory where they need the
loss (an allocator that forbids it, a runtime pool without scratch, a binding
with no device allocator): it keeps its scratch in a fixed library-owned
device array instead of a caller workspace. This file is collected last so a
failure here never hides the other tests. Each test checks the new entry
point, called through the C-ABI, against gh_ce_fwd_grad with a caller
workspace, on two calls in a row (the shared scratch keeps the previous
call's contents)."""

import numpy as np
import pytest
import torch

from greyhound_b200 import _lib
from greyhound_b200.testing import requires_gpu
from oracle import gh_oracle as O


def _call(noalloc: bool, x: torch.Tensor, t: torch.Tensor, mean: int, z: float):
    """One call of either entry point; returns (sums, gradient, lse) on the host."""
    lib = _lib.load()
    rows, V = x.shape
    code = _lib.dtype_code(x.dtype)
    grad = torch.empty_like(x)
    sums = [torch.empty((), dtype=torch.float32, device=x.device) for _ in range(3)]
    lse = torch.empty(rows, dtype=torch.float32, device=x.device)
    args_head = (x.data_ptr(), grad.data_ptr(), t.data_ptr(), rows, V, code, z, -100, mean, None,
                 sums[0].data_ptr(), sums[1].data_ptr(), sums[2].data_ptr(), lse.data_ptr())
    if noalloc:
        st = lib.gh_ce_fwd_grad_noalloc(*args_head, _lib.stream_of(x))
    else:
        ws = _lib.workspace(lib.gh_ce_workspace_bytes(rows, V, code), x.device)
        st = lib.gh_ce_fwd_grad(*args_head, ws.data_ptr(), ws.numel(), _lib.stream_of(x))
    _lib.check(st, "ce")
    torch.cuda.synchronize()
    return [s.item() for s in sums], grad.float().cpu(), lse.cpu()


@requires_gpu
@pytest.mark.parametrize("rows,V", [(16, 128256), (512, 32000), (37, 257)])
def test_noalloc_matches_workspace_entry_point_twice(rows, V):
    dev = torch.device("cuda", 0)
    for call, (seed, mean, z) in enumerate([(rows, 1, 1e-4), (rows + 1, 0, 0.0)]):
        x, t = O.make_ce_inputs(rows, V, seed, ignore_frac=0.2)
        xd = torch.from_numpy(x).to(dev, torch.bfloat16)
        td = torch.from_numpy(t).to(dev)
        ref_sums, ref_grad, ref_lse = _call(False, xd, td, mean, z)
        got_sums, got_grad, got_lse = _call(True, xd, td, mean, z)
        # loss within 1e-3 relative, gradient max-abs within 2e-2 of the max
        for a, b in zip(got_sums, ref_sums):
            assert abs(a - b) <= 1e-3 * max(1.0, abs(b)), (call, got_sums, ref_sums)
        assert (got_grad - ref_grad).abs().max() <= 2e-2 * ref_grad.abs().max()
        assert torch.allclose(got_lse, ref_lse, rtol=1e-5, atol=1e-5)
        assert got_sums[2] == float((t != -100).sum())


@requires_gpu
def test_noalloc_rejects_shapes_beyond_its_scratch():
    lib = _lib.load()
    cap = lib.gh_ce_noalloc_scratch_bytes()
    rows = 2 * cap // 12  # the per-row scratch alone exceeds the fixed array
    assert lib.gh_ce_workspace_bytes(rows, 64, _lib.GH_BF16) > cap
    dev = torch.device("cuda", 0)
    d = torch.empty(16, device=dev)
    st = lib.gh_ce_fwd_grad_noalloc(d.data_ptr(), None, d.data_ptr(), rows, 64, _lib.GH_BF16, 0.0, -100, 0, None,
                                    d.data_ptr(), d.data_ptr(), d.data_ptr(), None, _lib.stream_of(d))
    assert st == _lib.GH_EWORKSPACE  # the code gh_ce_fwd_grad gives a too-small workspace
    with pytest.raises(RuntimeError, match="scratch"):
        _lib.check(st, "noalloc")


def _rows_at_cap(lib, V: int, code: int) -> int:
    """The largest row count whose scratch still fits the fixed array."""
    cap = lib.gh_ce_noalloc_scratch_bytes()
    lo, hi = 0, 1 << 24
    while hi - lo > 1:
        mid = (lo + hi) // 2
        if lib.gh_ce_workspace_bytes(mid, V, code) <= cap:
            lo = mid
        else:
            hi = mid
    return lo


@requires_gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
def test_noalloc_at_the_scratch_limit(dtype):
    """Rows chosen so the scratch need sits just under the fixed size: the
    call is accepted and matches the workspace entry point; one row more is
    rejected."""
    lib = _lib.load()
    code = _lib.dtype_code(dtype)
    V = 64
    rows = _rows_at_cap(lib, V, code)
    assert lib.gh_ce_workspace_bytes(rows + 1, V, code) > lib.gh_ce_noalloc_scratch_bytes()
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(7)
    x = torch.randn(rows, V, device=dev, generator=g).to(dtype)
    t = torch.randint(0, V, (rows,), device=dev, generator=g)
    t[::17] = -100
    for mean in (1, 0):
        ref_sums, ref_grad, ref_lse = _call(False, x, t, mean, 1e-4)
        got_sums, got_grad, got_lse = _call(True, x, t, mean, 1e-4)
        for a, b in zip(got_sums, ref_sums):
            assert abs(a - b) <= 1e-3 * max(1.0, abs(b))
        assert (got_grad - ref_grad).abs().max() <= 2e-2 * ref_grad.abs().max()
        assert torch.allclose(got_lse, ref_lse, rtol=1e-5, atol=1e-5)
    t1 = torch.zeros(rows + 1, dtype=torch.int64, device=dev)
    x1 = torch.zeros(rows + 1, V, device=dev, dtype=dtype)
    st = lib.gh_ce_fwd_grad_noalloc(x1.data_ptr(), None, t1.data_ptr(), rows + 1, V, code, 0.0, -100, 0, None,
                                    x1.data_ptr(), x1.data_ptr(), x1.data_ptr(), None, _lib.stream_of(x1))
    assert st == _lib.GH_EWORKSPACE


@requires_gpu
def test_noalloc_zero_rows_gives_zero_sums():
    dev = torch.device("cuda", 0)
    x = torch.empty(0, 1000, device=dev, dtype=torch.bfloat16)
    t = torch.empty(0, dtype=torch.int64, device=dev)
    for _ in range(2):
        sums, _, _ = _call(True, x, t, 1, 0.0)
        assert sums == [0.0, 0.0, 0.0]


@requires_gpu
def test_noalloc_bad_label_status_is_readable():
    """The status word lives in the library-owned scratch; gh_ce_noalloc_status
    reads it (with a stream sync), so a label outside [0, V) is visible to a
    caller of this path too, and a clean call that follows clears it."""
    import ctypes

    lib = _lib.load()
    dev = torch.device("cuda", 0)
    x = torch.randn(4, 100, device=dev, dtype=torch.bfloat16)
    out = ctypes.c_int(-1)
    for labels, expect in (([1, 200, -100, 3], _lib.GH_DEV_BAD_LABEL), ([1, 2, -100, 3], 0)):
        t = torch.tensor(labels, device=dev)
        sums, grad, _ = _call(True, x, t, 1, 0.0)
        assert all(np.isfinite(sums))
        assert lib.gh_ce_noalloc_status(ctypes.byref(out), _lib.stream_of(x)) == _lib.GH_OK
        assert out.value == expect
        if expect:
            assert torch.all(grad[1] == 0)  # the bad row is treated as ignored
