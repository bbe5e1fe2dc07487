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
        if mode == "rows":
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
        torch.cuda.synchronize()
        out_q.put((rank, loss.item(), Hl.grad.float().cpu(), Wl.grad.float().cpu(), s, e))
        dist.destroy_process_group()
    except Exception:
        out_q.put((rank, "error", traceback.format_exc()))
