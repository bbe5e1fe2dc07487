"""Standalone cross-entropy on the GPU.

The first five tests restate src/tests/nn/functional/cross_entropy_test.py
(same shapes, tolerances, ignore patterns). The rest compare the CUDA path
with the CPU oracle (oracle/gh_oracle.py) on seeded inputs, against the golden
fixtures, and at the full workload size through properties."""

from typing import Literal

import numpy as np
import pytest
import torch
from torch import Tensor
from torch.library import opcheck

from greyhound_b200 import _lib
from greyhound_b200.kernels.cross_entropy import cross_entropy_with_grad, cross_entropy_with_grad_kernel
from greyhound_b200.nn.functional import cross_entropy
from greyhound_b200.ops.cross_entropy import cross_entropy_fwd, cross_entropy_fwd_mean
from greyhound_b200.testing import requires_gpu
from greyhound_b200.utils import get_default_device
from oracle import gh_oracle as O


def reference_cross_entropy(logits, target, ignore_index=-100, reduction="mean", z_loss_multiplier=0.0):
    logits = logits.float()
    ce_loss = torch.nn.functional.cross_entropy(logits, target, ignore_index=ignore_index, reduction=reduction)
    if z_loss_multiplier == 0.0:
        return ce_loss
    valid = target != ignore_index
    z_sum = torch.logsumexp(logits, dim=-1).square()[valid].sum()
    z_loss = z_loss_multiplier * z_sum
    if reduction == "mean":
        z_loss = z_loss / valid.sum().clamp(min=1)
    return ce_loss + z_loss


@requires_gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32, torch.float16])
@pytest.mark.parametrize("reduction", ["sum", "mean"])
@pytest.mark.parametrize("z_loss_multiplier", [0.0, 1e-4])
def test_cross_entropy_correctness_and_grad(dtype, reduction, z_loss_multiplier):
    device = get_default_device()
    batch_size, vocab_size = 37, 257
    logits = torch.randn(batch_size, vocab_size, device=device, dtype=dtype, requires_grad=True)
    target = torch.randint(0, vocab_size, (batch_size,), device=device)
    target[::5] = -100
    logits_ref = logits.detach().clone().requires_grad_(True)
    result = cross_entropy(logits, target, reduction=reduction, z_loss_multiplier=z_loss_multiplier)
    expected = reference_cross_entropy(logits_ref, target, reduction=reduction, z_loss_multiplier=z_loss_multiplier)
    assert torch.allclose(result.float(), expected.float(), rtol=5e-3, atol=5e-3)
    result.backward()
    expected.backward()
    rel = (logits.grad.float() - logits_ref.grad.float()).norm() / logits_ref.grad.float().norm()
    tol = 5e-3 if dtype is torch.float32 else 5e-2
    assert rel < tol


@requires_gpu
def test_cross_entropy_does_not_mutate_logits():
    device = get_default_device()
    logits = torch.randn(8, 97, device=device, dtype=torch.bfloat16, requires_grad=True)
    original = logits.detach().clone()
    target = torch.randint(0, logits.shape[-1], (logits.shape[0],), device=device)
    cross_entropy(logits, target).backward()
    assert torch.equal(logits.detach(), original)


@requires_gpu
def test_cross_entropy_fwd_returns_logits_gradient():
    device = get_default_device()
    logits = torch.randn(16, 257, device=device, dtype=torch.bfloat16)
    target = torch.randint(0, logits.shape[-1], (logits.shape[0],), device=device)
    target[::4] = -100
    logits_ref = logits.detach().clone().float().requires_grad_(True)
    ce_sum, z_sum, n_valid, grad_logits = cross_entropy_fwd(logits, target, 1e-4, -100)
    expected = reference_cross_entropy(logits_ref, target, reduction="sum", z_loss_multiplier=1e-4)
    expected.backward()
    assert torch.allclose((ce_sum + 1e-4 * z_sum).float(), expected.detach(), rtol=5e-3, atol=5e-3)
    assert n_valid.item() == float((target != -100).sum().item())
    assert torch.allclose(grad_logits.float(), logits_ref.grad, rtol=5e-3, atol=5e-3)


@requires_gpu
def test_cross_entropy_fwd_opcheck():
    device = get_default_device()
    logits = torch.randn(8, 256, device=device, dtype=torch.bfloat16)
    target = torch.randint(0, logits.shape[-1], (logits.shape[0],), device=device)
    opcheck(cross_entropy_fwd, (logits, target, 0.0, -100), raise_exception=True)
    opcheck(cross_entropy_fwd, (logits, target, 1e-4, -100), raise_exception=True)
    opcheck(cross_entropy_fwd_mean, (logits, target, 1e-4, -100), raise_exception=True)


@requires_gpu
@pytest.mark.parametrize("z_loss_multiplier", [0.0, 1e-4])
def test_cross_entropy_compile(z_loss_multiplier):
    device = get_default_device()
    logits = torch.randn(16, 257, device=device, dtype=torch.bfloat16)
    target = torch.randint(0, logits.shape[-1], (logits.shape[0],), device=device)

    @torch.compile(fullgraph=True)
    def compiled_fn(logits, target):
        return cross_entropy(logits, target, z_loss_multiplier=z_loss_multiplier)

    result = compiled_fn(logits, target)
    expected = reference_cross_entropy(logits, target, z_loss_multiplier=z_loss_multiplier)
    assert torch.allclose(result.float(), expected.float(), rtol=5e-3, atol=5e-3)


# --------------------------------------------------------------------------- oracle parity

def _dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.to(dtype)
    return t.to(get_default_device())


@requires_gpu
@pytest.mark.parametrize("name,rows,V,seed", [("ce37x257", 37, 257, 11), ("ce16x257", 16, 257, 12), ("ce64x4099", 64, 4099, 13)])
@pytest.mark.parametrize("red", ["sum", "mean"])
@pytest.mark.parametrize("z", [0.0, 1e-4])
def test_cross_entropy_matches_golden(golden, name, rows, V, seed, red, z):
    x, t = O.make_ce_inputs(rows, V, seed, ignore_frac=0.2)
    logits = _dev(x, torch.bfloat16).requires_grad_(True)
    target = _dev(t)
    loss = cross_entropy(logits, target, reduction=red, z_loss_multiplier=z)
    ref = float(golden[f"{name}/{red}/z{z}/loss"])
    assert abs(loss.item() - ref) <= 1e-3 * max(1.0, abs(ref))  # 1e-3 relative
    loss.backward()
    g = logits.grad.float().cpu().numpy()
    key = f"{name}/{red}/z{z}"
    gref = golden[f"{key}/grad"] if f"{key}/grad" in golden.files else None
    if gref is None:
        g = g.reshape(-1)[golden[f"{key}/grad_sel"]]
        gref = golden[f"{key}/grad_vals"]
    # bf16 gradient: max-abs <= 2e-2 after normalising by the max |reference|
    assert np.abs(g - gref).max() <= 2e-2 * max(np.abs(gref).max(), 1e-12)
    # ignore_index masking is exact
    if f"{key}/grad" in golden.files:
        assert np.all(logits.grad.float().cpu().numpy()[t == -100] == 0)


@requires_gpu
@pytest.mark.parametrize("rows,V", [(1, 1), (1, 7), (3, 8), (5, 9), (2, 2049), (17, 128256), (300, 4099), (0, 64)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_cross_entropy_with_grad_edge_shapes(rows, V, dtype):
    rng = np.random.default_rng(rows * 1000 + V)
    x = (rng.standard_normal((rows, V)) * 2).astype(np.float32)
    t = rng.integers(0, V, size=rows).astype(np.int64)
    if rows > 2:
        t[::3] = -100
    xd = _dev(x, dtype)
    xr = xd.float().cpu().numpy()
    td = _dev(t)
    grad = torch.empty_like(xd)
    ce, z, n = cross_entropy_with_grad(xd, td, 1e-4, -100, grad)
    rce, rz, rn, rg = O.cross_entropy_with_grad(xr, t, 1e-4, -100)
    assert n.item() == rn
    assert abs(ce.item() - rce) <= 1e-3 * max(1.0, abs(rce))
    assert abs(z.item() - rz) <= 1e-3 * max(1.0, abs(rz))
    if rows:
        np.testing.assert_allclose(grad.float().cpu().numpy(), rg, atol=2e-2 * max(np.abs(rg).max(), 1e-6), rtol=0)


@requires_gpu
def test_in_place_kernel_matches_out_of_place():
    x, t = O.make_ce_inputs(300, 5003, 7)
    xd = _dev(x, torch.bfloat16)
    td = _dev(t)
    g = torch.empty_like(xd)
    a = cross_entropy_with_grad(xd, td, 1e-4, -100, g)
    xin = xd.clone()
    b = cross_entropy_with_grad_kernel(xin, td, 1e-4, -100)
    assert torch.equal(xin, g)
    assert all(torch.equal(u, v) for u, v in zip(a, b))


@requires_gpu
def test_deterministic_loss_reduction():
    x, t = O.make_ce_inputs(512, 32000, 3)
    xd = _dev(x, torch.bfloat16)
    td = _dev(t)
    outs = [cross_entropy_with_grad(xd, td, 1e-4, -100, None) for _ in range(3)]
    for o in outs[1:]:
        assert all(torch.equal(a, b) for a, b in zip(o, outs[0]))


@requires_gpu
def test_bad_label_is_flagged_not_trapped():
    xd = torch.randn(4, 100, device=get_default_device(), dtype=torch.bfloat16)
    td = torch.tensor([1, 200, -100, 3], device=xd.device)
    lib = _lib.load()
    ws = _lib.workspace(lib.gh_ce_workspace_bytes(4, 100, _lib.GH_BF16), xd.device)
    out = torch.empty(3, device=xd.device)
    st = lib.gh_ce_fwd_grad(xd.data_ptr(), None, td.data_ptr(), 4, 100, _lib.GH_BF16, 0.0, -100, 0, None,
                            out[0:].data_ptr(), out[1:].data_ptr(), out[2:].data_ptr(), None,
                            ws.data_ptr(), ws.numel(), _lib.stream_of(xd))
    _lib.check(st, "ce")
    assert _lib.device_status(ws) & _lib.GH_DEV_BAD_LABEL
    assert torch.isfinite(out).all()


@requires_gpu
@pytest.mark.parametrize("rows", [16, 4096])
def test_cfg2_full_size_properties(rows):
    """Workload cfg2 ([4096, 128256] and [16, 128256] bf16) at full size.

    Properties: every valid gradient row sums to ~0 (softmax - onehot), ignored
    rows are exactly zero, and a sample of rows matches the oracle."""
    V = 128256
    x, t = O.make_ce_inputs(rows, V, 1)
    xd = _dev(x, torch.bfloat16)
    td = _dev(t)
    g = torch.empty_like(xd)
    ce, z, n = cross_entropy_with_grad(xd, td, 0.0, -100, g, mean_reduction=True)
    valid = td != -100
    assert n.item() == valid.sum().item()
    row_sums = g.float().sum(-1)
    assert torch.all(row_sums[valid].abs() < 2e-2 / max(n.item(), 1.0) * 8)
    assert torch.all(g[~valid] == 0)
    sample = np.arange(0, rows, max(1, rows // 16))
    rce, rz, rn, rg = O.cross_entropy_with_grad(x[sample], t[sample], 0.0, -100)
    gs = g[torch.from_numpy(sample).to(xd.device)].float().cpu().numpy()
    np.testing.assert_allclose(gs, rg / max(n.item(), 1.0), atol=2e-2 * np.abs(rg).max() / max(n.item(), 1.0))
    # loss sum vs oracle on the full tensor: chunked numpy in float64
    tot = 0.0
    for s in range(0, rows, 512):
        c, _, _, _ = O.cross_entropy_with_grad(x[s:s + 512], t[s:s + 512], 0.0, -100)
        tot += c
    assert abs(ce.item() - tot) <= 1e-3 * abs(tot)


@requires_gpu
def test_check_mode_raises_on_bad_label(monkeypatch):
    """GREYHOUND_B200_CHECK=1 turns the device status word into an exception."""
    monkeypatch.setattr(_lib, "CHECK_STATUS", True)
    x = torch.randn(4, 100, device=get_default_device(), dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="outside"):
        cross_entropy(x, torch.tensor([1, 200, -100, 3], device=x.device))
    assert cross_entropy(x, torch.tensor([1, 2, -100, 3], device=x.device)).isfinite()
