"""Generic chunked linear loss (bring-your-own loss-and-gradient callback).

Mirrors src/greyhound/ops/chunked_linear_loss.py: the chunk heuristic
(:24-48), the row-chunk loop ``logits -> callback -> grad_input, grad_weight``
(:56-103), the forward-only loop (:106-129) and ``ChunkedLinearLossFunction``
(:132-166). The callback is arbitrary Python, so this path stays a Python loop
around device GEMMs: for bf16 / fp16 operands these are the tcgen05 GEMMs of
the C-ABI (``gh_gemm``: logits, ``dH = dlogits W``, ``dW += dlogits^T H`` with
the accumulation done in the GEMM epilogue); fp32 operands use cuBLAS.
"""

from __future__ import annotations

from collections.abc import Callable

import torch
from torch import Tensor

from greyhound_b200.kernels.gemm import gemm_nt, gemm_nt_fp32
from greyhound_b200.kernels.linear_cross_entropy import chunk_size_for
from greyhound_b200.ops.scale import scale_by

__all__ = ["ChunkedLinearLossFunction"]

_chunked_linear_loss_chunk_size = chunk_size_for


def _resolve_chunk_size(B: int, D: int, V: int, element_size: int, chunk_size: int | None) -> int:
    if chunk_size is None:
        return chunk_size_for(B, D, V, element_size)
    if chunk_size <= 0:
        raise ValueError(f"chunk_size must be positive, got {chunk_size}")
    return min(chunk_size, B)


def _check_scalar_loss(loss: Tensor) -> None:
    if loss.ndim != 0:
        raise ValueError(f"chunked loss function must return a scalar tensor, got {loss.shape}")


def _check_grad_shape(grad_logits: Tensor, logits: Tensor) -> None:
    if grad_logits.shape != logits.shape:
        raise ValueError(
            f"loss gradient shape must match logits shape {tuple(logits.shape)}, "
            f"got {tuple(grad_logits.shape)}"
        )


def _tc_ok(inputs: Tensor, weight: Tensor) -> bool:
    return (
        inputs.is_cuda
        and inputs.dtype in (torch.bfloat16, torch.float16)
        and weight.dtype == inputs.dtype
        and inputs.shape[1] % 8 == 0
    )


def _logits(input_chunk: Tensor, weight: Tensor) -> Tensor:
    """``input_chunk @ weight`` ([D, V] operand): tcgen05 GEMM for bf16/fp16."""
    if _tc_ok(input_chunk, weight):
        return gemm_nt(input_chunk, weight.T)
    if _fp32_ok(input_chunk, weight):
        return gemm_nt_fp32(input_chunk, weight.T)
    return input_chunk @ weight


def _fp32_ok(*ts: Tensor) -> bool:
    """fp32 CUDA operands: the fp32 GEMMs emulated on the bf16 tcgen05 GEMM."""
    return all(t.is_cuda and t.dtype == torch.float32 for t in ts)


def _padded_grad(grad_logits: Tensor, dtype: torch.dtype) -> Tensor:
    """The callback's gradient as a [C, V] view with a 16-byte row pitch (TMA operand)."""
    C, V = grad_logits.shape
    ld = (V + 7) // 8 * 8
    if grad_logits.dtype == dtype and grad_logits.stride() == (ld, 1) and grad_logits.data_ptr() % 16 == 0:
        return grad_logits
    buf = torch.empty((C, ld), dtype=dtype, device=grad_logits.device)
    view = buf[:, :V]
    view.copy_(grad_logits)
    return view


def _chunked_linear_loss_with_grad(
    inputs: Tensor,
    weight: Tensor,
    loss_and_grad_fn: Callable[[Tensor, int, int], tuple[Tensor, Tensor]],
    fp32_grad_weight_accum: bool,
    chunk_size: int | None = None,
) -> tuple[Tensor, Tensor, Tensor]:
    """Loop of ``logits = x @ weight`` ([D, V] layout), callback, ``dH``/``dW`` updates."""
    B, D = inputs.shape
    V = weight.shape[1]
    chunk_size = _resolve_chunk_size(B, D, V, inputs.element_size(), chunk_size)
    loss_total = torch.zeros([], dtype=torch.float32, device=inputs.device)
    acc_dtype = torch.float32 if fp32_grad_weight_accum else weight.dtype
    tc = _tc_ok(inputs, weight)
    if tc:
        grad_input = torch.empty_like(inputs)
        # [V, D] row-major accumulator: returned as the [D, V] view (W.grad layout)
        grad_weight_accum = torch.empty([V, D], dtype=acc_dtype, device=weight.device)
    else:
        grad_input = torch.zeros_like(inputs)
        grad_weight_accum = torch.zeros([D, V], dtype=acc_dtype, device=weight.device)
    for start in range(0, B, chunk_size):
        end = min(start + chunk_size, B)
        input_chunk = inputs[start:end]
        logits_chunk = _logits(input_chunk, weight)
        loss_chunk, grad_logits = loss_and_grad_fn(logits_chunk, start, end)
        _check_scalar_loss(loss_chunk)
        _check_grad_shape(grad_logits, logits_chunk)
        loss_total = loss_total + loss_chunk.detach().float()
        grad_logits = grad_logits.detach()
        if tc:
            g = _padded_grad(grad_logits, inputs.dtype)
            gemm_nt(g, weight, out=grad_input[start:end])  # dlogits [C,V] . W [V,D]
            gemm_nt(g.T, input_chunk.T, out=grad_weight_accum,
                    addend=None if start == 0 else grad_weight_accum)
        elif _fp32_ok(inputs, weight) and acc_dtype == torch.float32:
            g = grad_logits.float()
            grad_input[start:end] = gemm_nt_fp32(g, weight)
            gemm_nt_fp32(input_chunk.T, g.T, out=grad_weight_accum, addend=grad_weight_accum)
        else:
            grad_input[start:end] = grad_logits @ weight.T
            torch.addmm(
                grad_weight_accum, input_chunk.T, grad_logits, out=grad_weight_accum, out_dtype=acc_dtype
            )
    if tc:
        return loss_total, grad_input, grad_weight_accum.to(weight.dtype).T
    return loss_total, grad_input, grad_weight_accum.to(weight.dtype)


def _chunked_linear_loss_forward_only(
    inputs: Tensor,
    weight: Tensor,
    loss_and_grad_fn: Callable[[Tensor, int, int], tuple[Tensor, Tensor]],
    chunk_size: int | None = None,
) -> Tensor:
    B, D = inputs.shape
    V = weight.shape[1]
    chunk_size = _resolve_chunk_size(B, D, V, inputs.element_size(), chunk_size)
    loss_total = torch.zeros([], dtype=torch.float32, device=inputs.device)
    for start in range(0, B, chunk_size):
        end = min(start + chunk_size, B)
        logits_chunk = _logits(inputs[start:end], weight)
        loss_chunk, grad_logits = loss_and_grad_fn(logits_chunk, start, end)
        _check_scalar_loss(loss_chunk)
        _check_grad_shape(grad_logits, logits_chunk)
        loss_total = loss_total + loss_chunk.detach().float()
    return loss_total


class ChunkedLinearLossFunction(torch.autograd.Function):
    @staticmethod
    def forward(
        ctx: object,
        inputs: Tensor,
        weight: Tensor,
        loss_and_grad_fn: Callable[[Tensor, int, int], tuple[Tensor, Tensor]],
        chunk_size: int | None = None,
        fp32_grad_weight_accum: bool = True,
    ) -> Tensor:
        if not ctx.needs_input_grad[0] and not ctx.needs_input_grad[1]:  # type: ignore[attr-defined]
            return _chunked_linear_loss_forward_only(inputs, weight, loss_and_grad_fn, chunk_size)
        loss, grad_input, grad_weight = _chunked_linear_loss_with_grad(
            inputs, weight, loss_and_grad_fn, fp32_grad_weight_accum, chunk_size
        )
        ctx.save_for_backward(grad_input, grad_weight)  # type: ignore[attr-defined]
        return loss

    @staticmethod
    def backward(ctx: object, grad_output: Tensor):  # type: ignore[override]
        grad_input, grad_weight = ctx.saved_tensors  # type: ignore[attr-defined]
        return scale_by(grad_input, grad_output), scale_by(grad_weight, grad_output), None, None, None
