"""Worker processes for the multi-GPU (NCCL) tests: real kernels, one process
per GPU. Test infrastructure only."""

from __future__ import annotations

import datetime
import os
import traceback

import torch
import torch.distributed as dist


def _init(rank, world, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))


def worker(rank, world, port, data, mode, out_q):
    try:
        _init(rank, world, port)
        from greyhound_b200.distributed import (
            row_sharded_linear_cross_entropy,
            shard_range,
            vocab_sharded_linear_cross_entropy,
        )

        H, W, t, red, z = data
        dev = torch.device("cuda", rank)
        if mode == "rows_nccl":  # the NCCL all-reduce path instead of the fused band exchange
            os.environ["GREYHOUND_B200_DP_PEER"] = "0"
        if mode in ("rows", "rows_nccl"):
            s, e = shard_range(H.shape[0], rank, world)
            Hl = H[s:e].to(dev).requires_grad_(True)
            Wl = W.to(dev).requires_grad_(True)
            loss = row_sharded_linear_cross_entropy(Hl, Wl, t[s:e].to(dev), reduction=red, z_loss_multiplier=z)
        else:
            s, e = shard_range(W.shape[0], rank, world)
            Hl = H.to(dev).requires_grad_(True)
            Wl = W[s:e].to(dev).requires_grad_(True)
            loss = vocab_sharded_linear_cross_entropy(Hl, Wl, t.to(dev), s, reduction=red, z_loss_multiplier=z)
        loss.backward()
        if mode == "rows":  # a second step reuses the exchange buffers
            Hl.grad = None
            Wl.grad = None
            loss = row_sharded_linear_cross_entropy(Hl, Wl, t[s:e].to(dev), reduction=red, z_loss_multiplier=z)
            loss.backward()
        torch.cuda.synchronize()
        out_q.put((rank, loss.item(), Hl.grad.float().cpu(), Wl.grad.float().cpu(), s, e))
        dist.destroy_process_group()
    except Exception:
        out_q.put((rank, "error", traceback.format_exc()))


def worker_vocab_shard_check(rank, world, port, shape, out_q):
    """Vocab-parallel linear CE at a given shape, checked inside the worker
    against fp32 torch of the reference semantics (the full weight is rebuilt
    from its seed on every rank); returns only error figures."""
    try:
        _init(rank, world, port)
        from greyhound_b200.distributed import shard_range, vocab_sharded_linear_cross_entropy

        N, D, V = shape
        dev = torch.device("cuda", rank)
        g = torch.Generator(device=dev).manual_seed(4)
        H = torch.randn(N, D, device=dev, generator=g).bfloat16()
        W = (torch.randn(V, D, device=dev, generator=g) * 0.015).bfloat16()
        t = torch.randint(0, V, (N,), device=dev, generator=g)
        t[torch.rand(N, device=dev, generator=g) < 0.02] = -100
        s, e = shard_range(V, rank, world)
        Hl = H.clone().requires_grad_(True)
        Wl = W[s:e].clone().requires_grad_(True)
        loss = vocab_sharded_linear_cross_entropy(Hl, Wl, t, s)
        loss.backward()
        valid = t != -100
        n = valid.sum().float()
        lse = torch.empty(N, device=dev)
        ref_loss = torch.zeros((), device=dev, dtype=torch.float64)
        for r0 in range(0, N, 4096):
            x = (H[r0:r0 + 4096] @ W.T).float()
            lse[r0:r0 + 4096] = torch.logsumexp(x, -1)
            tc = t[r0:r0 + 4096]
            ref_loss += torch.where(tc != -100, lse[r0:r0 + 4096] - x.gather(1, tc.clamp(min=0)[:, None])[:, 0],
                                    0.0).double().sum()
            del x
        ref_loss = (ref_loss / n).item()

        def dl(rows_idx, c0, c1):
            x = (H[rows_idx] @ W[c0:c1].T).float()
            p = torch.exp(x - lse[rows_idx][:, None])
            tt = t[rows_idx]
            hit = (tt >= c0) & (tt < c1)
            p[hit.nonzero()[:, 0], tt[hit] - c0] -= 1.0
            p[tt == -100] = 0.0
            return p.bfloat16().float() / n

        rows = torch.arange(0, N, 1021, device=dev)
        ref_dH = dl(rows, 0, V) @ W.float()
        err_h = ((Hl.grad[rows].float() - ref_dH).abs().max() / ref_dH.abs().max()).item()
        band = (s, min(s + 256, e))
        ref_dW = torch.zeros(band[1] - band[0], D, device=dev)
        for r0 in range(0, N, 8192):
            ref_dW += dl(torch.arange(r0, r0 + 8192, device=dev), *band).T @ H[r0:r0 + 8192].float()
        err_w = ((Wl.grad[: band[1] - band[0]].float() - ref_dW).abs().max() / ref_dW.abs().max()).item()
        out_q.put((rank, loss.item(), ref_loss, err_h, err_w))
        dist.destroy_process_group()
    except Exception:
        out_q.put((rank, "error", traceback.format_exc()))
