"""Chunked linear cross-entropy custom op + autograd Function.

Mirrors src/greyhound/ops/chunked_linear_cross_entropy.py: the op
``greyhound::chunked_linear_cross_entropy_fwd(inputs[B,D], weight[D,V], target[B],
z_loss_multiplier, fp32_grad_weight_accum, ignore_index=-100)
-> (ce_sum, z_sum, n_valid, grad_input[B,D], grad_weight[D,V])`` (:19-67) with
its fake (:70-88), the forward-only fast path (:91-132) and
``ChunkedLinearCrossEntropyFunction`` (:135-185), including the
``ctx.needs_input_grad`` gate (:150) and gradients computed in the forward and
scaled by ``grad_output`` in the backward.

B200 differences (results unchanged within tolerance): ``grad_weight`` is
returned as the transposed view of a row-major ``[V, D]`` buffer (strides
``(1, D)``) instead of a contiguous ``[D, V]`` tensor (:87), so ``W.grad`` of
the ``[V, D]`` parameter is produced without a 1 GB re-layout copy; and for
``reduction="mean"``
the Function calls ``greyhound::chunked_linear_cross_entropy_fwd_mean``, which
folds ``1 / max(n_valid, 1)`` into the logits gradient before the two
gradient GEMMs instead of two ``mul_`` passes over ``grad_input`` and
``grad_weight`` afterwards (:159-164).
"""

from __future__ import annotations

from typing import Literal

import torch
from torch import Tensor

from greyhound_b200.ops.scale import scale_by
from greyhound_b200.kernels.linear_cross_entropy import (
    lce_workspace_bytes,
    linear_cross_entropy_grads_from,
    linear_cross_entropy_loss,
    linear_cross_entropy_stats_keep,
    linear_cross_entropy_with_grad,
    two_phase_ok,
)

__all__ = [
    "ChunkedLinearCrossEntropyFunction",
    "chunked_linear_cross_entropy_fwd",
    "chunked_linear_cross_entropy_fwd_mean",
    "chunked_linear_cross_entropy_loss",
    "chunked_linear_cross_entropy_stats",
    "chunked_linear_cross_entropy_grads",
]


def _fake(inputs: Tensor, weight: Tensor) -> tuple[Tensor, Tensor, Tensor, Tensor, Tensor]:
    B, D = inputs.shape
    V = weight.shape[1]
    return (
        torch.empty([], dtype=torch.float32, device=inputs.device),
        torch.empty([], dtype=torch.float32, device=inputs.device),
        torch.empty([], dtype=torch.float32, device=inputs.device),
        torch.empty([B, D], dtype=inputs.dtype, device=inputs.device),
        # [D, V] gradient stored as a transposed [V, D] row-major buffer
        torch.empty_strided([D, V], [1, D], dtype=weight.dtype, device=inputs.device),
    )


@torch.library.custom_op("greyhound::chunked_linear_cross_entropy_fwd", mutates_args=())
def chunked_linear_cross_entropy_fwd(
    inputs: Tensor,  # [B, D]
    weight: Tensor,  # [D, V]
    target: Tensor,  # [B]
    z_loss_multiplier: float,
    fp32_grad_weight_accum: bool,
    ignore_index: int = -100,
) -> tuple[Tensor, Tensor, Tensor, Tensor, Tensor]:
    """Returns (ce_sum, z_sum, n_valid, grad_input, grad_weight) of the summed loss."""
    return linear_cross_entropy_with_grad(
        inputs, weight, target, z_loss_multiplier, fp32_grad_weight_accum, ignore_index
    )


@chunked_linear_cross_entropy_fwd.register_fake
def _(
    inputs: Tensor,
    weight: Tensor,
    target: Tensor,
    z_loss_multiplier: float,
    fp32_grad_weight_accum: bool,
    ignore_index: int = -100,
) -> tuple[Tensor, Tensor, Tensor, Tensor, Tensor]:
    return _fake(inputs, weight)


@torch.library.custom_op("greyhound::chunked_linear_cross_entropy_fwd_mean", mutates_args=())
def chunked_linear_cross_entropy_fwd_mean(
    inputs: Tensor,
    weight: Tensor,
    target: Tensor,
    z_loss_multiplier: float,
    fp32_grad_weight_accum: bool,
    ignore_index: int = -100,
) -> tuple[Tensor, Tensor, Tensor, Tensor, Tensor]:
    """As ``chunked_linear_cross_entropy_fwd`` with gradients divided by max(n_valid, 1)."""
    return linear_cross_entropy_with_grad(
        inputs,
        weight,
        target,
        z_loss_multiplier,
        fp32_grad_weight_accum,
        ignore_index,
        mean_reduction=True,
    )


@chunked_linear_cross_entropy_fwd_mean.register_fake
def _(
    inputs: Tensor,
    weight: Tensor,
    target: Tensor,
    z_loss_multiplier: float,
    fp32_grad_weight_accum: bool,
    ignore_index: int = -100,
) -> tuple[Tensor, Tensor, Tensor, Tensor, Tensor]:
    return _fake(inputs, weight)


@torch.library.custom_op("greyhound::chunked_linear_cross_entropy_loss", mutates_args=())
def chunked_linear_cross_entropy_loss(
    inputs: Tensor,
    weight: Tensor,
    target: Tensor,
    z_loss_multiplier: float,
    ignore_index: int = -100,
) -> tuple[Tensor, Tensor, Tensor]:
    """Forward-only sums (ce_sum, z_sum, n_valid); no gradient buffers."""
    return linear_cross_entropy_loss(inputs, weight, target, z_loss_multiplier, ignore_index)


@chunked_linear_cross_entropy_loss.register_fake
def _(
    inputs: Tensor,
    weight: Tensor,
    target: Tensor,
    z_loss_multiplier: float,
    ignore_index: int = -100,
) -> tuple[Tensor, Tensor, Tensor]:
    return _fake(inputs, weight)[:3]


@torch.library.custom_op("greyhound::chunked_linear_cross_entropy_stats", mutates_args=())
def chunked_linear_cross_entropy_stats(
    inputs: Tensor,
    weight: Tensor,
    target: Tensor,
    z_loss_multiplier: float,
    fp32_grad_weight_accum: bool,
    ignore_index: int,
    mean_reduction: bool,
) -> tuple[Tensor, Tensor, Tensor, Tensor]:
    """(ce_sum, z_sum, n_valid, workspace): the loss of the single-chunk
    training path with everything the two gradient GEMMs need kept in the
    workspace (uint8) for ``chunked_linear_cross_entropy_grads``."""
    return linear_cross_entropy_stats_keep(inputs, weight, target, z_loss_multiplier, fp32_grad_weight_accum,
                                           ignore_index, mean_reduction)


@chunked_linear_cross_entropy_stats.register_fake
def _(inputs, weight, target, z_loss_multiplier, fp32_grad_weight_accum, ignore_index, mean_reduction):
    f = _fake(inputs, weight)
    ws = torch.empty(lce_workspace_bytes(inputs, weight, fp32_grad_weight_accum), dtype=torch.uint8,
                     device=inputs.device)
    return f[0], f[1], f[2], ws


@torch.library.custom_op("greyhound::chunked_linear_cross_entropy_grads", mutates_args=())
def chunked_linear_cross_entropy_grads(
    workspace: Tensor,
    inputs: Tensor,
    weight: Tensor,
    grad_output: Tensor,
    fp32_grad_weight_accum: bool,
) -> tuple[Tensor, Tensor]:
    """(grad_input [B, D], grad_weight [D, V]) times grad_output, from the
    workspace of ``chunked_linear_cross_entropy_stats``."""
    return linear_cross_entropy_grads_from(workspace, inputs, weight, fp32_grad_weight_accum, grad_output)


@chunked_linear_cross_entropy_grads.register_fake
def _(workspace, inputs, weight, grad_output, fp32_grad_weight_accum):
    f = _fake(inputs, weight)
    return f[3], f[4]


def _forward_only_chunked_ce(
    inputs: Tensor,
    weight: Tensor,
    target: Tensor,
    ignore_index: int,
    reduction: str,
    z_loss_multiplier: float,
) -> Tensor:
    """Forward-only path (no gradient buffers), ops/chunked_linear_cross_entropy.py:91-132."""
    ce_sum, z_sum, n_valid = chunked_linear_cross_entropy_loss(
        inputs, weight, target, z_loss_multiplier, ignore_index
    )
    loss = ce_sum + z_loss_multiplier * z_sum
    if reduction == "mean":
        loss = loss / n_valid.clamp(min=1.0)
    return loss


class ChunkedLinearCrossEntropyFunction(torch.autograd.Function):
    @staticmethod
    def forward(
        ctx: object,
        inputs: Tensor,  # [B, D]
        weight: Tensor,  # [D, V]
        target: Tensor,  # [B]
        ignore_index: int = -100,
        reduction: Literal["sum", "mean"] = "mean",
        z_loss_multiplier: float = 0.0,
        fp32_grad_weight_accum: bool = True,
    ) -> Tensor:
        # torch.is_grad_enabled() is always False inside Function.forward; gate on
        # needs_input_grad exactly like the reference (:150).
        if not ctx.needs_input_grad[0] and not ctx.needs_input_grad[1]:  # type: ignore[attr-defined]
            return _forward_only_chunked_ce(
                inputs, weight, target, ignore_index, reduction, z_loss_multiplier
            )
        if reduction not in ("mean", "sum"):
            raise ValueError(f"Unsupported reduction: {reduction}")
        if two_phase_ok(inputs, weight):
            # loss now, gradients in the backward already multiplied by
            # grad_output: no scaling pass, and a second backward through a
            # retained graph recomputes them with its own grad_output
            ce_sum, z_sum, n_valid, ws = chunked_linear_cross_entropy_stats(
                inputs, weight, target, z_loss_multiplier, fp32_grad_weight_accum, ignore_index,
                reduction == "mean"
            )
            loss = ce_sum + z_loss_multiplier * z_sum
            if reduction == "mean":
                loss = loss / n_valid.clamp(min=1.0)
            ctx.two_phase = True  # type: ignore[attr-defined]
            ctx.fp32_accum = fp32_grad_weight_accum  # type: ignore[attr-defined]
            ctx.save_for_backward(ws, inputs, weight)  # type: ignore[attr-defined]
            return loss
        ctx.two_phase = False  # type: ignore[attr-defined]
        if reduction == "mean":
            ce_sum, z_sum, n_valid, grad_input, grad_weight = chunked_linear_cross_entropy_fwd_mean(
                inputs, weight, target, z_loss_multiplier, fp32_grad_weight_accum, ignore_index
            )
            loss = (ce_sum + z_loss_multiplier * z_sum) / n_valid.clamp(min=1.0)
        elif reduction == "sum":
            ce_sum, z_sum, n_valid, grad_input, grad_weight = chunked_linear_cross_entropy_fwd(
                inputs, weight, target, z_loss_multiplier, fp32_grad_weight_accum, ignore_index
            )
            loss = ce_sum + z_loss_multiplier * z_sum
        else:
            raise ValueError(f"Unsupported reduction: {reduction}")
        ctx.save_for_backward(grad_input, grad_weight, n_valid)  # type: ignore[attr-defined]
        return loss

    @staticmethod
    def backward(ctx: object, grad_output: Tensor):  # type: ignore[override]
        if ctx.two_phase:  # type: ignore[attr-defined]
            ws, inputs, weight = ctx.saved_tensors  # type: ignore[attr-defined]
            gi, gw = chunked_linear_cross_entropy_grads(ws, inputs, weight, grad_output,
                                                        ctx.fp32_accum)  # type: ignore[attr-defined]
            return gi, gw, None, None, None, None, None
        grad_input, grad_weight, _ = ctx.saved_tensors  # type: ignore[attr-defined]
        return (
            scale_by(grad_input, grad_output),
            scale_by(grad_weight, grad_output),
            None,
            None,
            None,
            None,
            None,
        )
