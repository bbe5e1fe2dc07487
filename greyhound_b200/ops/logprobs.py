"""Selective log-softmax custom ops + autograd Function.

Mirrors src/greyhound/ops/logprobs.py: same op
``greyhound::selective_log_softmax_fwd(logits, index) -> Tensor`` with the same
fake (output in the logits dtype, ops/logprobs.py:11-18). The reference's
backward raises NotImplementedError (ops/logprobs.py:30); here it is
implemented: the forward also keeps the per-row logsumexp
(``greyhound::selective_log_softmax_fwd_lse``) and the backward runs
``greyhound::selective_log_softmax_bwd``.
"""

from __future__ import annotations

from typing import Any

import torch
from torch import Tensor

from greyhound_b200.kernels.logprobs import (
    selective_log_softmax_backward_kernel,
    selective_log_softmax_kernel,
    selective_log_softmax_with_lse,
)

__all__ = [
    "SelectiveLogSoftmaxFunction",
    "selective_log_softmax_fwd",
    "selective_log_softmax_fwd_lse",
    "selective_log_softmax_bwd",
]


@torch.library.custom_op("greyhound::selective_log_softmax_fwd", mutates_args=())
def selective_log_softmax_fwd(logits: Tensor, index: Tensor) -> Tensor:
    return selective_log_softmax_kernel(logits, index)


@selective_log_softmax_fwd.register_fake
def _(logits: Tensor, index: Tensor) -> Tensor:
    return torch.empty_like(index, dtype=logits.dtype, device=logits.device)


@torch.library.custom_op("greyhound::selective_log_softmax_fwd_lse", mutates_args=())
def selective_log_softmax_fwd_lse(logits: Tensor, index: Tensor) -> tuple[Tensor, Tensor]:
    out, lse = selective_log_softmax_with_lse(logits, index, want_lse=True)
    assert lse is not None
    return out, lse


@selective_log_softmax_fwd_lse.register_fake
def _(logits: Tensor, index: Tensor) -> tuple[Tensor, Tensor]:
    return (
        torch.empty_like(index, dtype=logits.dtype, device=logits.device),
        torch.empty_like(index, dtype=torch.float32, device=logits.device),
    )


@torch.library.custom_op("greyhound::selective_log_softmax_bwd", mutates_args=())
def selective_log_softmax_bwd(logits: Tensor, index: Tensor, lse: Tensor, grad_out: Tensor) -> Tensor:
    return selective_log_softmax_backward_kernel(logits, index, lse, grad_out)


@selective_log_softmax_bwd.register_fake
def _(logits: Tensor, index: Tensor, lse: Tensor, grad_out: Tensor) -> Tensor:
    return torch.empty_like(logits)


class SelectiveLogSoftmaxFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx: Any, logits: Tensor, index: Tensor) -> Tensor:
        if not ctx.needs_input_grad[0]:
            return selective_log_softmax_fwd(logits, index)
        out, lse = selective_log_softmax_fwd_lse(logits, index)
        ctx.save_for_backward(logits, index, lse)
        return out

    @staticmethod
    def backward(ctx: Any, grad_out: Tensor) -> tuple[Tensor | None, None]:  # type: ignore[override]
        logits, index, lse = ctx.saved_tensors
        return selective_log_softmax_bwd(logits, index, lse, grad_out), None
