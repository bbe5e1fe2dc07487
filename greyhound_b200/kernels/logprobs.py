"""Selective log-softmax row kernels (sm_100a, via the C-ABI).

Drop-in for ``greyhound.kernels.logprobs`` (src/greyhound/kernels/logprobs.py):
``selective_log_softmax_kernel`` keeps the reference signature, validation and
output dtype (the logits dtype, kernels/logprobs.py:131-172). The backward
kernel is new: the reference has none (ops/logprobs.py:30).
"""

from __future__ import annotations

import torch
from torch import Tensor

from greyhound_b200 import _lib

__all__ = [
    "selective_log_softmax_kernel",
    "selective_log_softmax_with_lse",
    "selective_log_softmax_backward_kernel",
]


def _validate(logits: Tensor, index: Tensor) -> None:
    # Same checks and messages as kernels/logprobs.py:138-153.
    if logits.ndim < 2:
        raise ValueError(f"expected logits with at least 2 dimensions, got {logits.ndim}")
    if index.shape != logits.shape[:-1]:
        raise ValueError(
            f"expected index shape {tuple(logits.shape[:-1])}, got {tuple(index.shape)}"
        )
    if not logits.is_cuda or index.device != logits.device:
        raise ValueError("expected logits and index on the same CUDA device")
    if logits.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        raise TypeError(f"unsupported logits dtype: {logits.dtype}")
    if index.dtype not in (torch.int32, torch.int64):
        raise TypeError(f"expected int32 or int64 index, got {index.dtype}")
    if logits.shape[-1] <= 0:
        raise ValueError("expected non-empty vocabulary dimension")
    if not logits.is_contiguous() or not index.is_contiguous():
        raise ValueError("expected contiguous logits and index")


def selective_log_softmax_with_lse(
    logits: Tensor,
    index: Tensor,
    out_dtype: torch.dtype | None = None,
    want_lse: bool = True,
) -> tuple[Tensor, Tensor | None]:
    """``gather(log_softmax(logits), index)`` plus the per-row logsumexp (fp32)."""
    _validate(logits, index)
    vocab = logits.shape[-1]
    rows = index.numel()
    out_dtype = logits.dtype if out_dtype is None else out_dtype
    out = torch.empty(index.shape, dtype=out_dtype, device=logits.device)
    lse = torch.empty(index.shape, dtype=torch.float32, device=logits.device) if want_lse else None
    lib = _lib.load()
    _lib.raise_pending(logits.device, "selective_log_softmax")
    code = _lib.dtype_code(logits.dtype)
    ws = _lib.workspace(lib.gh_sls_workspace_bytes(rows, vocab, code), logits.device)
    status = lib.gh_sls_fwd(
        logits.data_ptr(),
        index.data_ptr(),
        _lib.dtype_code(index.dtype),
        rows,
        vocab,
        code,
        out.data_ptr(),
        _lib.dtype_code(out_dtype),
        _lib.ptr(lse),
        ws.data_ptr(),
        ws.numel(),
        _lib.stream_of(logits),
    )
    _lib.check(status, "selective_log_softmax")
    _lib.raise_on_status(ws, "selective_log_softmax")
    return out, lse


def selective_log_softmax_kernel(logits: Tensor, index: Tensor) -> Tensor:
    """Compute ``gather(log_softmax(logits, -1), index)`` without materializing logprobs.

    ``logits`` is flattened over every leading dimension and reduced row-by-row
    across the final vocabulary dimension with an fp32 online log-sum-exp; one
    selected log-probability is written per row, in the logits dtype.
    """
    out, _ = selective_log_softmax_with_lse(logits, index, want_lse=False)
    return out


def selective_log_softmax_backward_kernel(
    logits: Tensor, index: Tensor, lse: Tensor, grad_out: Tensor
) -> Tensor:
    """d/dlogits of ``sum(grad_out * selective_log_softmax(logits, index))``.

    ``grad[r, v] = grad_out[r] * ([v == index[r]] - exp(logits[r, v] - lse[r]))``.
    """
    _validate(logits, index)
    if lse.shape != index.shape or lse.dtype != torch.float32:
        raise ValueError("lse must be fp32 with the index shape")
    grad_out = grad_out.contiguous()
    if grad_out.shape != index.shape:
        raise ValueError(f"expected grad_out shape {tuple(index.shape)}, got {tuple(grad_out.shape)}")
    if grad_out.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        grad_out = grad_out.float()
    grad = torch.empty_like(logits)
    lib = _lib.load()
    _lib.raise_pending(logits.device, "selective_log_softmax_backward")
    status = lib.gh_sls_bwd(
        logits.data_ptr(),
        index.data_ptr(),
        _lib.dtype_code(index.dtype),
        lse.contiguous().data_ptr(),
        grad_out.data_ptr(),
        _lib.dtype_code(grad_out.dtype),
        index.numel(),
        logits.shape[-1],
        _lib.dtype_code(logits.dtype),
        grad.data_ptr(),
        _lib.stream_of(logits),
    )
    _lib.check(status, "selective_log_softmax_backward")
    return grad
