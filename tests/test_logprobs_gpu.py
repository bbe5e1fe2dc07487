"""Selective log-softmax on the GPU: restates src/tests/nn/functional/logprobs_test.py
and adds oracle/golden parity, the (new) backward, and full-size properties."""

import numpy as np
import pytest
import torch
from torch.library import opcheck

from greyhound_b200.kernels.logprobs import selective_log_softmax_with_lse
from greyhound_b200.nn.functional import selective_log_softmax
from greyhound_b200.ops.logprobs import (
    selective_log_softmax_bwd,
    selective_log_softmax_fwd,
    selective_log_softmax_fwd_lse,
)
from greyhound_b200.testing import requires_gpu
from greyhound_b200.utils import get_default_device
from oracle import gh_oracle as O


def reference_selective_log_softmax(logits, index):
    logprobs = logits.log_softmax(dim=-1)
    return torch.gather(logprobs, dim=-1, index=index.unsqueeze(-1)).squeeze(-1)


@requires_gpu
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
def test_selective_log_softmax_correctness(dtype):
    device = get_default_device()
    logits = torch.randn(4, 16, 257, device=device, dtype=dtype)
    index = torch.randint(0, logits.shape[-1], logits.shape[:-1], device=device)
    result = selective_log_softmax(logits, index)
    expected = reference_selective_log_softmax(logits, index)
    assert result.shape == index.shape
    assert result.dtype == logits.dtype
    assert torch.allclose(result.float(), expected.float(), rtol=5e-3, atol=5e-3)


@requires_gpu
@pytest.mark.parametrize("index_dtype", [torch.int32, torch.int64])
def test_selective_log_softmax_index_dtypes(index_dtype):
    device = get_default_device()
    logits = torch.randn(8, 513, device=device, dtype=torch.bfloat16)
    index = torch.randint(0, logits.shape[-1], logits.shape[:-1], device=device, dtype=index_dtype)
    result = selective_log_softmax(logits, index)
    expected = reference_selective_log_softmax(logits, index.long())
    assert torch.allclose(result.float(), expected.float(), rtol=5e-3, atol=5e-3)


@requires_gpu
def test_selective_log_softmax_fwd_opcheck():
    device = get_default_device()
    logits = torch.randn(4, 16, 256, device=device, dtype=torch.bfloat16)
    index = torch.randint(0, logits.shape[-1], logits.shape[:-1], device=device)
    opcheck(selective_log_softmax_fwd, (logits, index), raise_exception=True)
    opcheck(selective_log_softmax_fwd_lse, (logits, index), raise_exception=True)
    lse = torch.logsumexp(logits.float(), -1)
    g = torch.randn(index.shape, device=device)
    opcheck(selective_log_softmax_bwd, (logits, index, lse, g), raise_exception=True)


@requires_gpu
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
def test_selective_log_softmax_backward(dtype):
    device = get_default_device()
    logits = torch.randn(4, 16, 257, device=device, dtype=dtype, requires_grad=True)
    index = torch.randint(0, logits.shape[-1], logits.shape[:-1], device=device)
    ref = logits.detach().float().clone().requires_grad_(True)
    g = torch.randn(index.shape, device=device)
    (selective_log_softmax(logits, index).float() * g).sum().backward()
    (reference_selective_log_softmax(ref, index) * g).sum().backward()
    rel = (logits.grad.float() - ref.grad).norm() / ref.grad.norm()
    assert rel < (5e-3 if dtype is torch.float32 else 5e-2)


@requires_gpu
def test_selective_log_softmax_compile():
    device = get_default_device()
    logits = torch.randn(16, 257, device=device, dtype=torch.bfloat16)
    index = torch.randint(0, 257, (16,), device=device)

    @torch.compile(fullgraph=True)
    def f(x, i):
        return selective_log_softmax(x, i)

    assert torch.allclose(f(logits, index).float(), reference_selective_log_softmax(logits.float(), index), rtol=5e-3, atol=5e-3)


def _dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.to(dtype)
    return t.to(get_default_device())


@requires_gpu
@pytest.mark.parametrize("name,shape,seed", [("sls4x16x257", (4, 16, 257), 21), ("sls8x513", (8, 513), 22), ("sls16x151936", (16, 151936), 23)])
def test_selective_log_softmax_matches_golden(golden, name, shape, seed):
    rows = int(np.prod(shape[:-1]))
    x, idx = O.make_sls_inputs(rows, shape[-1], seed)
    xd = _dev(x.reshape(shape), torch.bfloat16).requires_grad_(True)
    idd = _dev(idx.reshape(shape[:-1]))
    out, lse = selective_log_softmax_with_lse(xd.detach(), idd, out_dtype=torch.float32)
    ref = golden[f"{name}/out"]
    np.testing.assert_allclose(out.cpu().numpy(), ref, rtol=1e-3, atol=1e-3 * np.abs(ref).max())
    gout = _dev(golden[f"{name}/grad_out"])
    (selective_log_softmax(xd, idd).float() * gout).sum().backward()
    g = xd.grad.float().cpu().numpy()
    if f"{name}/grad" in golden.files:
        gref = golden[f"{name}/grad"]
    else:
        g = g.reshape(-1)[golden[f"{name}/grad_sel"]]
        gref = golden[f"{name}/grad_vals"]
    assert np.abs(g - gref).max() <= 2e-2 * np.abs(gref).max()


@requires_gpu
@pytest.mark.parametrize("rows,V", [(1, 1), (3, 7), (5, 9), (300, 4099), (7, 151936), (1024, 151936)])
def test_selective_log_softmax_edge_shapes(rows, V):
    x, idx = O.make_sls_inputs(rows, V, rows + V)
    xd = _dev(x, torch.bfloat16)
    out, lse = selective_log_softmax_with_lse(xd, _dev(idx), out_dtype=torch.float32)
    ref = O.selective_log_softmax(xd.float().cpu().numpy(), idx)
    np.testing.assert_allclose(out.cpu().numpy(), ref, rtol=1e-4, atol=1e-3)
    np.testing.assert_allclose(lse.cpu().numpy(), O.logsumexp_rows(xd.float().cpu().numpy()), rtol=1e-5, atol=1e-4)


@requires_gpu
def test_cfg4_full_size_properties():
    """cfg4: [65536, 151936] bf16 logits (19.9 GB). Checks on sampled rows
    against the oracle, plus backward properties: each gradient row sums to 0
    and gradient[r, index[r]] = g (1 - p)."""
    rows, V = 65536, 151936
    dev = get_default_device()
    gen = torch.Generator(device=dev)
    gen.manual_seed(3)
    xd = (torch.randn(rows, V, device=dev, generator=gen) * 3).to(torch.bfloat16)
    idx = torch.randint(0, V, (rows,), device=dev, generator=gen)
    out, lse = selective_log_softmax_with_lse(xd, idx, out_dtype=torch.float32)
    sample = torch.arange(0, rows, 4093, device=dev)
    xs = xd[sample].float().cpu().numpy()
    ref = O.selective_log_softmax(xs, idx[sample].cpu().numpy())
    np.testing.assert_allclose(out[sample].cpu().numpy(), ref, rtol=1e-4, atol=1e-3)
    # backward on a 4096-row slice (the full-size gradient would need another 19.9 GB)
    sl = slice(0, 4096)
    g = torch.randn(4096, device=dev, generator=gen)
    grad = selective_log_softmax_bwd(xd[sl], idx[sl], lse[sl], g)
    row_sum = grad.float().sum(-1)
    assert torch.all(row_sum.abs() < 2e-2 * (g.abs() + 1e-3) + 1e-3)
    p_idx = torch.exp(out[sl].double())
    at_idx = grad[torch.arange(4096, device=dev), idx[sl]].double()
    assert torch.allclose(at_idx, (g.double() * (1 - p_idx)), rtol=1e-2, atol=1e-2)
    del xd
