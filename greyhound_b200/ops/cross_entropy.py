"""Cross-entropy custom op + autograd Function.

Mirrors src/greyhound/ops/cross_entropy.py: same op name and schema
``greyhound::cross_entropy_fwd(logits, target, z_loss_multiplier, ignore_index=-100)
-> (ce_sum, z_sum, n_valid, grad_logits)`` (ops/cross_entropy.py:11-26) with
the same fake (:29-42) and the same Function semantics (:45-85).

B200 differences (results unchanged): the gradient is written straight into a
fresh buffer instead of cloning the logits first (ops/cross_entropy.py:19),
and for ``reduction="mean"`` a second op, ``greyhound::cross_entropy_fwd_mean``,
folds ``1 / max(n_valid, 1)`` into that write instead of a separate ``mul_``
pass (:63-66).
"""

from __future__ import annotations

from typing import Any, Literal

import torch
from torch import Tensor

from greyhound_b200.ops.scale import scale_by
from greyhound_b200.kernels.cross_entropy import cross_entropy_with_grad

__all__ = ["CrossEntropyFunction", "cross_entropy_fwd", "cross_entropy_fwd_mean"]


def _fake(logits: Tensor) -> tuple[Tensor, Tensor, Tensor, Tensor]:
    return (
        torch.empty([], dtype=torch.float32, device=logits.device),
        torch.empty([], dtype=torch.float32, device=logits.device),
        torch.empty([], dtype=torch.float32, device=logits.device),
        torch.empty_like(logits),
    )


@torch.library.custom_op("greyhound::cross_entropy_fwd", mutates_args=())
def cross_entropy_fwd(
    logits: Tensor,
    target: Tensor,
    z_loss_multiplier: float,
    ignore_index: int = -100,
) -> tuple[Tensor, Tensor, Tensor, Tensor]:
    """Cross-entropy forward that also returns the (sum-reduction) logits gradient."""
    grad_logits = torch.empty_like(logits, memory_format=torch.contiguous_format)
    ce_sum, z_sum, n_valid = cross_entropy_with_grad(
        logits, target, z_loss_multiplier, ignore_index, grad_logits
    )
    return ce_sum, z_sum, n_valid, grad_logits


@cross_entropy_fwd.register_fake
def _(
    logits: Tensor,
    target: Tensor,
    z_loss_multiplier: float,
    ignore_index: int = -100,
) -> tuple[Tensor, Tensor, Tensor, Tensor]:
    del target, z_loss_multiplier, ignore_index
    return _fake(logits)


@torch.library.custom_op("greyhound::cross_entropy_fwd_mean", mutates_args=())
def cross_entropy_fwd_mean(
    logits: Tensor,
    target: Tensor,
    z_loss_multiplier: float,
    ignore_index: int = -100,
) -> tuple[Tensor, Tensor, Tensor, Tensor]:
    """As ``cross_entropy_fwd`` but the gradient is divided by ``max(n_valid, 1)``."""
    grad_logits = torch.empty_like(logits, memory_format=torch.contiguous_format)
    ce_sum, z_sum, n_valid = cross_entropy_with_grad(
        logits, target, z_loss_multiplier, ignore_index, grad_logits, mean_reduction=True
    )
    return ce_sum, z_sum, n_valid, grad_logits


@cross_entropy_fwd_mean.register_fake
def _(
    logits: Tensor,
    target: Tensor,
    z_loss_multiplier: float,
    ignore_index: int = -100,
) -> tuple[Tensor, Tensor, Tensor, Tensor]:
    del target, z_loss_multiplier, ignore_index
    return _fake(logits)


class CrossEntropyFunction(torch.autograd.Function):
    @staticmethod
    def forward(
        ctx: Any,
        logits: Tensor,
        target: Tensor,
        ignore_index: int = -100,
        reduction: Literal["sum", "mean"] = "mean",
        z_loss_multiplier: float = 0.0,
    ) -> Tensor:
        if reduction == "mean":
            ce_sum, z_sum, n_valid, grad_logits = cross_entropy_fwd_mean(
                logits, target, z_loss_multiplier, ignore_index
            )
            loss = (ce_sum + z_loss_multiplier * z_sum) / n_valid.clamp(min=1.0)
        elif reduction == "sum":
            ce_sum, z_sum, n_valid, grad_logits = cross_entropy_fwd(
                logits, target, z_loss_multiplier, ignore_index
            )
            loss = ce_sum + z_loss_multiplier * z_sum
        else:
            raise ValueError(f"Unsupported reduction: {reduction}")
        ctx.save_for_backward(grad_logits)
        return loss

    @staticmethod
    def backward(ctx: Any, grad_output: Tensor) -> tuple[Tensor, None, None, None, None]:  # type: ignore[override]
        (grad_logits,) = ctx.saved_tensors
        return scale_by(grad_logits, grad_output), None, None, None, None
