"""Multi-GPU layer: data-parallel row sharding and vocab-parallel sharding of the
chunked linear cross-entropy (one process per GPU, ``torch.distributed``; NCCL
on GPUs, Gloo for CPU tests of the sharding arithmetic).

The reference is single-device only (src/greyhound/utils.py:4-7); these modes
are new. Both keep the reference's loss semantics: the loss is the sum over
all valid tokens of all ranks, divided by the *global* valid-token count for
``reduction="mean"``.

* Row sharding (``RowShardedLinearCrossEntropy``): each rank holds its own rows
  of ``inputs``/``target`` and a replica of ``weight``. One scalar all-reduce
  gives the global valid count before any gradient is written, so the
  ``1 / n_global`` scale is folded into the logits gradient; the weight
  gradient is then summed across ranks with one all-reduce.
* Vocab sharding (``VocabShardedLinearCrossEntropy``): each rank holds rows
  ``[r*V/P, (r+1)*V/P)`` of ``weight`` and all rows of ``inputs``. Per row the
  ranks exchange (max, sum-exp, target-logit) with one all-gather, combine them
  into the exact global logsumexp, then each writes its slice of the logits
  gradient, its weight-gradient shard (no communication) and a partial input
  gradient that is summed with one all-reduce.
"""

from __future__ import annotations

from typing import Literal

import torch
import torch.distributed as dist
from torch import Tensor

from greyhound_b200.ops.scale import scale_by
from greyhound_b200.kernels import linear_cross_entropy as lce

__all__ = [
    "row_sharded_linear_cross_entropy",
    "vocab_sharded_linear_cross_entropy",
    "combine_vocab_stats",
    "shard_range",
]


def shard_range(total: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous near-equal split of ``[0, total)``; the first ``total % world`` shards get one extra."""
    base, rem = divmod(total, world)
    start = rank * base + min(rank, rem)
    return start, start + base + (1 if rank < rem else 0)


def _global_scale(target: Tensor, ignore_index: int, reduction: str, group) -> tuple[Tensor, Tensor]:
    n = (target != ignore_index).sum().to(torch.float32).reshape(1)
    if dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(n, group=group)
    if reduction == "mean":
        scale = 1.0 / n.clamp(min=1.0)
    elif reduction == "sum":
        scale = torch.ones_like(n)
    else:
        raise ValueError(f"Unsupported reduction: {reduction}")
    return n.reshape(()), scale


class RowShardedLinearCrossEntropy(torch.autograd.Function):
    @staticmethod
    def forward(ctx, inputs, weight_dv, target, ignore_index, reduction, z_loss_multiplier, fp32_accum, group):
        n_global, scale = _global_scale(target, ignore_index, reduction, group)
        world = dist.get_world_size(group) if dist.is_initialized() else 1
        hook = None
        if world > 1:
            def hook(grad_weight: Tensor):
                return dist.all_reduce(grad_weight, group=group, async_op=True)
        ce, zs, _, gi, gw = lce.linear_cross_entropy_with_grad(
            inputs, weight_dv, target, z_loss_multiplier, fp32_accum, ignore_index,
            grad_scale=scale, grad_weight_hook=hook,
        )
        loss = (ce + z_loss_multiplier * zs).reshape(1)
        if world > 1:
            dist.all_reduce(loss, group=group)
        loss = (loss * scale).reshape(())
        ctx.save_for_backward(gi, gw)
        return loss

    @staticmethod
    def backward(ctx, g):
        gi, gw = ctx.saved_tensors
        return scale_by(gi, g), scale_by(gw, g), None, None, None, None, None, None


def row_sharded_linear_cross_entropy(
    inputs: Tensor,
    weight: Tensor,
    target: Tensor,
    ignore_index: int = -100,
    reduction: Literal["sum", "mean"] = "mean",
    z_loss_multiplier: float = 0.0,
    grad_weight_accum_dtype: Literal["fp32", "weight"] = "fp32",
    group=None,
) -> Tensor:
    """Data-parallel ``chunked_linear_cross_entropy``: this rank's rows, replicated ``weight [V, D]``.

    Returns the global loss (identical on every rank); ``weight.grad`` is the
    all-reduced global gradient, ``inputs.grad`` this rank's rows.
    """
    if grad_weight_accum_dtype not in ("fp32", "weight"):
        raise ValueError(f"grad_weight_accum_dtype must be either 'fp32' or 'weight', got {grad_weight_accum_dtype!r}")
    return RowShardedLinearCrossEntropy.apply(
        inputs, weight.T, target, ignore_index, reduction, z_loss_multiplier,
        grad_weight_accum_dtype == "fp32", group,
    )


def combine_vocab_stats(stats: Tensor) -> tuple[Tensor, Tensor]:
    """Combine per-shard row statistics into the global logsumexp and target logit.

    ``stats`` is ``[P, rows, 3]`` fp32 holding, for every vocab shard, the row
    max ``m``, ``s = sum exp(x - m)`` over the shard and the target logit (or
    ``-inf`` when the target is not in that shard). Exact, order-independent
    merge: ``lse = M + log(sum_p s_p exp(m_p - M))`` with ``M = max_p m_p``.
    """
    m, s, xt = stats[..., 0], stats[..., 1], stats[..., 2]
    M = m.max(dim=0).values
    Msafe = torch.where(torch.isfinite(M), M, torch.zeros_like(M))
    total = (s * torch.exp(m - Msafe)).sum(dim=0)
    lse = Msafe + torch.log(total)
    x_target = xt.max(dim=0).values
    return lse, x_target


class VocabShardedLinearCrossEntropy(torch.autograd.Function):
    @staticmethod
    def forward(ctx, inputs, weight_shard, target, vocab_start, ignore_index, reduction, z_loss_multiplier, group):
        world = dist.get_world_size(group) if dist.is_initialized() else 1
        valid = target != ignore_index
        n = valid.sum().to(torch.float32)
        if reduction == "mean":
            scale = 1.0 / n.clamp(min=1.0)
        elif reduction == "sum":
            scale = torch.ones_like(n)
        else:
            raise ValueError(f"Unsupported reduction: {reduction}")
        stats, state = lce.vocab_shard_stats(inputs, weight_shard, target, vocab_start)
        if world > 1:
            gathered = [torch.empty_like(stats) for _ in range(world)]
            dist.all_gather(gathered, stats, group=group)
            all_stats = torch.stack(gathered)
        else:
            all_stats = stats[None]
        lse, x_t = combine_vocab_stats(all_stats)
        ce = torch.where(valid, lse - x_t, torch.zeros_like(lse)).sum()
        zs = torch.where(valid, lse * lse, torch.zeros_like(lse)).sum()
        loss = (ce + z_loss_multiplier * zs) * scale
        hook = None
        if world > 1:
            def hook(gi_partial: Tensor):
                return dist.all_reduce(gi_partial, group=group, async_op=True)
        gi, gw = lce.vocab_shard_grads(
            inputs, weight_shard, state, target, vocab_start, lse, z_loss_multiplier, ignore_index, scale,
            grad_input_hook=hook,
        )
        ctx.save_for_backward(gi, gw)
        return loss

    @staticmethod
    def backward(ctx, g):
        gi, gw = ctx.saved_tensors
        return scale_by(gi, g), scale_by(gw, g), None, None, None, None, None, None


def vocab_sharded_linear_cross_entropy(
    inputs: Tensor,
    weight_shard: Tensor,
    target: Tensor,
    vocab_start: int,
    ignore_index: int = -100,
    reduction: Literal["sum", "mean"] = "mean",
    z_loss_multiplier: float = 0.0,
    group=None,
) -> Tensor:
    """Vocab-parallel ``chunked_linear_cross_entropy``.

    ``weight_shard`` is this rank's ``[V_local, D]`` rows of the ``[V, D]``
    weight, starting at vocab id ``vocab_start``; ``inputs``/``target`` are the
    full (replicated) rows. Returns the global loss on every rank;
    ``weight_shard.grad`` is this shard's gradient and ``inputs.grad`` the full
    (all-reduced) input gradient.
    """
    return VocabShardedLinearCrossEntropy.apply(
        inputs, weight_shard, target, int(vocab_start), ignore_index, reduction, z_loss_multiplier, group
    )
