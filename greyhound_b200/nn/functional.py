"""Public functional API — same signatures and semantics as src/greyhound/nn/functional.py.

``selective_log_softmax`` (:53-69), ``cross_entropy`` (:72-116),
``autograd_loss_and_logits_grad`` (:119-148), ``chunked_linear_loss`` (:151-223)
and ``chunked_linear_cross_entropy`` (:226-287). ``weight`` is ``[V, D]`` and is
handed to the ops as the ``[D, V]`` view ``weight.T``, exactly as the reference
does, so the op schemas and their fakes are unchanged.
"""

from __future__ import annotations

from collections.abc import Callable
from typing import Any, Literal, cast

import torch
from torch import Tensor

from greyhound_b200.ops.chunked_linear_cross_entropy import ChunkedLinearCrossEntropyFunction
from greyhound_b200.ops.chunked_linear_loss import ChunkedLinearLossFunction
from greyhound_b200.ops.cross_entropy import CrossEntropyFunction
from greyhound_b200.ops.logprobs import SelectiveLogSoftmaxFunction

__all__ = [
    "selective_log_softmax",
    "cross_entropy",
    "autograd_loss_and_logits_grad",
    "chunked_linear_loss",
    "chunked_linear_cross_entropy",
]


def _slice_chunk_arg(value: Any, start: int, end: int, batch_size: int) -> Any:
    if isinstance(value, Tensor) and value.ndim > 0 and value.shape[0] == batch_size:
        return value[start:end]
    return value


def _check_scalar_loss(loss: Tensor) -> None:
    if loss.ndim != 0:
        raise ValueError(f"chunked loss function must return a scalar tensor, got {loss.shape}")


def _check_accum_dtype(grad_weight_accum_dtype: str) -> None:
    if grad_weight_accum_dtype not in ("fp32", "weight"):
        raise ValueError(
            "grad_weight_accum_dtype must be either 'fp32' or 'weight', "
            f"got {grad_weight_accum_dtype!r}"
        )


def selective_log_softmax(logits: Tensor, index: Tensor) -> Tensor:
    """Log-probability of ``index`` under ``softmax(logits)`` along the last dim.

    Equivalent to ``gather(logits.log_softmax(-1), -1, index[..., None])[..., 0]``
    without materialising the log-probabilities: one streaming fp32
    log-sum-exp per row. Output has ``index``'s shape and the logits dtype.
    Differentiable with respect to ``logits``.
    """
    return cast(Tensor, SelectiveLogSoftmaxFunction.apply(logits, index))


def cross_entropy(
    logits: Tensor,
    target: Tensor,
    ignore_index: int = -100,
    reduction: Literal["sum", "mean"] = "mean",
    z_loss_multiplier: float = 0.0,
) -> Tensor:
    """Cross-entropy of materialised ``[B, V]`` logits, plus optional z-loss.

    ``loss = sum_valid(lse - logits[target]) + z_loss_multiplier * sum_valid(lse^2)``,
    divided by the number of valid (``target != ignore_index``) rows when
    ``reduction="mean"``. The logits gradient is produced in the same pass and
    returned by autograd; the input ``logits`` tensor is never modified.
    """
    return cast(
        Tensor,
        CrossEntropyFunction.apply(logits, target, ignore_index, reduction, z_loss_multiplier),
    )


def autograd_loss_and_logits_grad(
    loss_fn: Callable[..., Tensor],
) -> Callable[..., tuple[Tensor, Tensor]]:
    """Wrap a scalar loss ``loss_fn(logits, *args, **kwargs)`` to return ``(loss, dloss/dlogits)``."""

    def loss_and_grad(logits: Tensor, *args: Any, **kwargs: Any) -> tuple[Tensor, Tensor]:
        with torch.enable_grad():
            logits_for_grad = logits.detach().requires_grad_(True)
            loss = loss_fn(logits_for_grad, *args, **kwargs)
            _check_scalar_loss(loss)
            (grad_logits,) = torch.autograd.grad(loss, logits_for_grad)
        return loss.detach(), grad_logits.detach()

    return loss_and_grad


def chunked_linear_loss(
    inputs: Tensor,
    weight: Tensor,
    loss_and_grad_fn: Callable[..., tuple[Tensor, Tensor]],
    *loss_args: Any,
    chunk_size: int | None = None,
    grad_weight_accum_dtype: Literal["fp32", "weight"] = "fp32",
    **loss_kwargs: Any,
) -> Tensor:
    """Row-chunked ``inputs @ weight.T`` followed by a user loss-and-gradient callback.

    For each row chunk the callback gets ``(logits_chunk, *args, **kwargs)``,
    with every tensor argument whose leading dim equals ``inputs.shape[0]``
    sliced to the chunk's rows, and returns ``(scalar_loss, grad_logits)``.
    Input and weight gradients are accumulated chunk by chunk (weight gradient
    in fp32 unless ``grad_weight_accum_dtype="weight"``). Returns the summed loss.
    """
    _check_accum_dtype(grad_weight_accum_dtype)
    batch_size = inputs.shape[0]

    def chunk_loss_and_grad_fn(logits_chunk: Tensor, start: int, end: int) -> tuple[Tensor, Tensor]:
        chunk_args = tuple(_slice_chunk_arg(a, start, end, batch_size) for a in loss_args)
        chunk_kwargs = {k: _slice_chunk_arg(v, start, end, batch_size) for k, v in loss_kwargs.items()}
        return loss_and_grad_fn(logits_chunk, *chunk_args, **chunk_kwargs)

    return cast(
        Tensor,
        ChunkedLinearLossFunction.apply(
            inputs, weight.T, chunk_loss_and_grad_fn, chunk_size, grad_weight_accum_dtype == "fp32"
        ),
    )


def chunked_linear_cross_entropy(
    inputs: Tensor,
    weight: Tensor,
    target: Tensor,
    ignore_index: int = -100,
    reduction: Literal["sum", "mean"] = "mean",
    z_loss_multiplier: float = 0.0,
    grad_weight_accum_dtype: Literal["fp32", "weight"] = "fp32",
) -> Tensor:
    """Cross-entropy of ``inputs @ weight.T`` without keeping the logits.

    ``inputs`` is ``[BT, D]``, ``weight`` is ``[V, D]``, ``target`` is ``[BT]``
    with class ids in ``[0, V)`` or ``ignore_index``. The forward computes the
    loss and, when an input requires grad, both gradients; ``backward`` only
    scales them by the incoming gradient. ``grad_weight_accum_dtype="fp32"``
    accumulates the weight gradient in fp32 and casts once; ``"weight"``
    accumulates in the parameter dtype.
    """
    _check_accum_dtype(grad_weight_accum_dtype)
    return cast(
        Tensor,
        ChunkedLinearCrossEntropyFunction.apply(
            inputs,
            weight.T,
            target,
            ignore_index,
            reduction,
            z_loss_multiplier,
            grad_weight_accum_dtype == "fp32",
        ),
    )
