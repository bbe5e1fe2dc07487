"""Cross-entropy + logits-gradient row kernel (sm_100a, via the C-ABI).

Drop-in for ``greyhound.kernels.cross_entropy`` (src/greyhound/kernels/cross_entropy.py).
``cross_entropy_with_grad_kernel`` keeps the reference signature, validation
messages and in-place semantics (kernels/cross_entropy.py:166-204);
``cross_entropy_with_grad`` is the out-of-place form the ops layer uses.
"""

from __future__ import annotations

import torch
from torch import Tensor

from greyhound_b200 import _lib

__all__ = ["cross_entropy_with_grad_kernel", "cross_entropy_with_grad"]


def _validate(logits: Tensor, labels: Tensor) -> None:
    # Same checks and messages as kernels/cross_entropy.py:173-184.
    if logits.ndim != 2:
        raise ValueError(f"expected 2D logits, got shape {tuple(logits.shape)}")
    if labels.shape != (logits.shape[0],):
        raise ValueError(f"expected labels shape {(logits.shape[0],)}, got {tuple(labels.shape)}")
    if not logits.is_cuda or labels.device != logits.device:
        raise ValueError("expected logits and labels on the same CUDA device")
    if logits.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        raise TypeError(f"unsupported logits dtype: {logits.dtype}")
    if labels.dtype != torch.int64:
        raise TypeError(f"expected int64 labels, got {labels.dtype}")
    if not logits.is_contiguous() or not labels.is_contiguous():
        raise ValueError("expected contiguous logits and labels")


def cross_entropy_with_grad(
    logits: Tensor,
    labels: Tensor,
    z_loss_multiplier: float,
    ignore_index: int,
    grad_out: Tensor | None,
    mean_reduction: bool = False,
    lse_out: Tensor | None = None,
    grad_scale: Tensor | None = None,
) -> tuple[Tensor, Tensor, Tensor]:
    """Loss sums of ``logits`` and (optionally) its gradient written to ``grad_out``.

    ``grad_out`` may be ``logits`` itself (in place), a fresh tensor of the same
    shape and dtype, or None (loss only). With ``mean_reduction`` the gradient
    is already divided by ``max(n_valid, 1)``; ``grad_scale`` (a 1-element fp32
    device tensor) multiplies it further.
    Returns 0-d fp32 tensors ``(ce_sum, z_sum, n_valid)``.
    """
    _validate(logits, labels)
    if grad_out is not None:
        if grad_out.shape != logits.shape or grad_out.dtype != logits.dtype:
            raise ValueError("grad_out must match logits in shape and dtype")
        if not grad_out.is_contiguous() or grad_out.device != logits.device:
            raise ValueError("grad_out must be contiguous and on the logits device")
    rows, vocab = logits.shape
    if vocab <= 0:
        raise ValueError("expected non-empty vocabulary dimension")
    lib = _lib.load()
    dev = logits.device
    _lib.raise_pending(dev, "cross_entropy_with_grad")
    # Three separate 0-d tensors, like the reference (outputs never alias).
    ce_sum = torch.empty((), dtype=torch.float32, device=dev)
    z_sum = torch.empty((), dtype=torch.float32, device=dev)
    n_valid = torch.empty((), dtype=torch.float32, device=dev)
    code = _lib.dtype_code(logits.dtype)
    ws = _lib.workspace(lib.gh_ce_workspace_bytes(rows, vocab, code), dev)
    status = lib.gh_ce_fwd_grad(
        logits.data_ptr(),
        _lib.ptr(grad_out),
        labels.data_ptr(),
        rows,
        vocab,
        code,
        float(z_loss_multiplier),
        int(ignore_index),
        1 if mean_reduction else 0,
        _lib.ptr(grad_scale),
        ce_sum.data_ptr(),
        z_sum.data_ptr(),
        n_valid.data_ptr(),
        _lib.ptr(lse_out),
        ws.data_ptr(),
        ws.numel(),
        _lib.stream_of(logits),
    )
    _lib.check(status, "cross_entropy_with_grad")
    _lib.raise_on_status(ws, "cross_entropy_with_grad")
    return ce_sum, z_sum, n_valid


def cross_entropy_with_grad_kernel(
    logits: Tensor,
    labels: Tensor,
    z_loss_multiplier: float,
    ignore_index: int,
) -> tuple[Tensor, Tensor, Tensor]:
    """Compute summed losses and overwrite ``logits`` with its gradient."""
    return cross_entropy_with_grad(logits, labels, z_loss_multiplier, ignore_index, grad_out=logits)
