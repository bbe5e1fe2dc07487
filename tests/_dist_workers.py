"""Worker processes for the Gloo (CPU) tests of greyhound_b200.distributed.

The GPU kernels are replaced by plain-torch CPU stand-ins with the same
contracts, so these tests exercise only the host-side sharding logic: the
global valid-count all-reduce and mean scale, the weight-gradient all-reduce
hook, the vocab-shard statistics exchange and merge, and the input-gradient
all-reduce. Test infrastructure only."""

from __future__ import annotations

import os
import traceback

import torch
import torch.distributed as dist


def cpu_lce_with_grad(inputs, weight_dv, target, z, fp32_accum, ignore_index, mean_reduction=False,
                      grad_scale=None, grad_weight_hook=None):
    with torch.enable_grad():  # called inside autograd.Function.forward
        x = inputs.detach().float().requires_grad_(True)
        w = weight_dv.detach().float().requires_grad_(True)
        logits = x @ w
        valid = target != ignore_index
        lse = torch.logsumexp(logits, -1)
        xt = logits.gather(1, target.clamp(min=0)[:, None])[:, 0]
        ce = torch.where(valid, lse - xt, torch.zeros_like(lse)).sum()
        zs = torch.where(valid, lse * lse, torch.zeros_like(lse)).sum()
        n = valid.sum().float()
        gi, gw = torch.autograd.grad(ce + z * zs, [x, w])
    s = grad_scale.reshape(()) if grad_scale is not None else torch.tensor(1.0)
    if mean_reduction:
        s = s / n.clamp(min=1.0)
    gw_vd = (gw * s).T.contiguous().to(weight_dv.dtype)
    if grad_weight_hook is not None:
        work = grad_weight_hook(gw_vd)
        if work is not None:
            work.wait()
    return ce.detach(), zs.detach(), n.detach(), (gi * s).to(inputs.dtype), gw_vd.T


def cpu_vocab_shard_stats(inputs, weight_shard, target, vocab_start):
    logits = inputs.float() @ weight_shard.float().T
    lse = torch.logsumexp(logits, -1)
    Vs = weight_shard.shape[0]
    loc = target - vocab_start
    inside = (loc >= 0) & (loc < Vs)
    xt = logits.gather(1, loc.clamp(0, Vs - 1)[:, None])[:, 0]
    xt = torch.where(inside, xt, torch.full_like(xt, float("-inf")))
    return torch.stack([lse, torch.ones_like(lse), xt], 1), logits


def cpu_vocab_shard_grads(inputs, weight_shard, state, target, vocab_start, lse, z, ignore_index, scale,
                          grad_input_hook=None):
    logits = state
    Vs = weight_shard.shape[0]
    p = torch.exp(logits - lse[:, None]) * (1 + 2 * z * lse)[:, None]
    loc = target - vocab_start
    inside = (loc >= 0) & (loc < Vs) & (target != ignore_index)
    p[inside.nonzero()[:, 0], loc[inside]] -= 1.0
    p[target == ignore_index] = 0.0
    p = p * scale.reshape(())
    gi = (p @ weight_shard.float()).to(inputs.dtype)
    work = grad_input_hook(gi) if grad_input_hook is not None else None
    gw = (p.T @ inputs.float()).to(weight_shard.dtype)
    if work is not None:
        work.wait()
    return gi, gw


def _patch():
    import greyhound_b200.distributed as D
    import greyhound_b200.kernels.linear_cross_entropy as L

    L.linear_cross_entropy_with_grad = cpu_lce_with_grad
    L.vocab_shard_stats = cpu_vocab_shard_stats
    L.vocab_shard_grads = cpu_vocab_shard_grads
    D.scale_by = lambda t, g: t * g


def _init(rank, world, store_path):
    # file rendezvous: no TCP port to race for between concurrently started tests
    import datetime

    dist.init_process_group("gloo", init_method=f"file://{store_path}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=20))


def row_sharded_worker(rank, world, port, data, out_q):
    try:
        _init(rank, world, port)
        _patch()
        from greyhound_b200.distributed import row_sharded_linear_cross_entropy, shard_range

        H, W, t, red, z = data
        s, e = shard_range(H.shape[0], rank, world)
        Hl = H[s:e].clone().requires_grad_(True)
        Wl = W.clone().requires_grad_(True)
        loss = row_sharded_linear_cross_entropy(Hl, Wl, t[s:e], reduction=red, z_loss_multiplier=z)
        loss.backward()
        out_q.put((rank, loss.item(), Hl.grad.float(), Wl.grad.float(), s, e))
        dist.destroy_process_group()
    except Exception:
        out_q.put((rank, "error", traceback.format_exc()))


def vocab_sharded_worker(rank, world, port, data, out_q):
    try:
        _init(rank, world, port)
        _patch()
        from greyhound_b200.distributed import shard_range, vocab_sharded_linear_cross_entropy

        H, W, t, red, z = data
        vs, ve = shard_range(W.shape[0], rank, world)
        Hl = H.clone().requires_grad_(True)
        Ws = W[vs:ve].clone().requires_grad_(True)
        loss = vocab_sharded_linear_cross_entropy(Hl, Ws, t, vs, reduction=red, z_loss_multiplier=z)
        loss.backward()
        out_q.put((rank, loss.item(), Hl.grad.float(), Ws.grad.float(), vs, ve))
        dist.destroy_process_group()
    except Exception:
        out_q.put((rank, "error", traceback.format_exc()))


def dead_rank_worker(rank, world, port, data, out_q):
    """Rank 1 leaves before the first collective; rank 0 must get an error, not hang."""
    try:
        _init(rank, world, port)
        _patch()
        if rank == 1:
            out_q.put((rank, "left"))
            out_q.close()
            out_q.join_thread()  # flush before the abrupt exit
            os._exit(0)
        from greyhound_b200.distributed import row_sharded_linear_cross_entropy

        H, W, t, red, z = data
        try:
            row_sharded_linear_cross_entropy(H.clone().requires_grad_(True), W.clone().requires_grad_(True), t)
            out_q.put((rank, "no error"))
        except Exception as exc:  # expected: the collective fails (peer gone / timeout)
            out_q.put((rank, "detected", type(exc).__name__))
    except Exception:
        out_q.put((rank, "error", traceback.format_exc()))
