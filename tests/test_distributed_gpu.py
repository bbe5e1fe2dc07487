"""Row-sharded and vocab-parallel linear cross-entropy on 2 GPUs (NCCL, real
kernels) against the single-GPU result on the full data. Skipped with fewer
than 2 GPUs."""

import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from greyhound_b200.testing import requires_gpu
from oracle import gh_oracle as O

two_gpus = pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")


def _needs(n):
    return pytest.mark.skipif(torch.cuda.device_count() < n, reason=f"needs {n} GPUs")


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _run(data, mode, world=2):
    import _dist_gpu_workers as Wk

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=Wk.worker, args=(r, world, port, data, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    return sorted(out, key=lambda x: x[0])


def _maxabs_norm(a, ref):
    a = np.asarray(a, np.float64)
    ref = np.asarray(ref, np.float64)
    return np.abs(a - ref).max() / max(np.abs(ref).max(), 1e-30)


@requires_gpu
@two_gpus
@pytest.mark.parametrize("mode", ["rows", "rows_nccl", "vocab"])
@pytest.mark.parametrize("red", ["mean", "sum"])
def test_two_gpu_sharding_matches_oracle(mode, red):
    H, W, t = O.make_lce_inputs(1024, 512, 12000, 7, 0.05, 0.05)
    data = (torch.from_numpy(H).bfloat16(), torch.from_numpy(W).bfloat16(), torch.from_numpy(t), red, 1e-4)
    out = _run(data, mode)
    assert all(o[1] != "error" for o in out), out
    loss, dH, dW = O.chunked_linear_cross_entropy(H, W, t, -100, red, 1e-4)
    for rank, l, gH, gW, s, e in out:
        assert abs(l - loss) <= 1e-3 * abs(loss)
        if mode in ("rows", "rows_nccl"):
            assert _maxabs_norm(gH.numpy(), dH[s:e]) <= 2e-2
            assert _maxabs_norm(gW.numpy(), dW) <= 2e-2
        else:
            assert _maxabs_norm(gH.numpy(), dH) <= 2e-2
            assert _maxabs_norm(gW.numpy(), dW[s:e]) <= 2e-2


@requires_gpu
@pytest.mark.parametrize("world", [pytest.param(4, marks=_needs(4)), pytest.param(8, marks=_needs(8))])
def test_band_exchange_on_more_gpus(world):
    """The fused weight-gradient reduce-scatter with 4 and 8 ranks, on a
    vocabulary that does not divide into the bands evenly."""
    H, W, t = O.make_lce_inputs(256 * world, 256, 30011, 8, 0.05, 0.05)
    data = (torch.from_numpy(H).bfloat16(), torch.from_numpy(W).bfloat16(), torch.from_numpy(t), "mean", 0.0)
    out = _run(data, "rows", world)
    assert all(o[1] != "error" for o in out), out
    loss, dH, dW = O.chunked_linear_cross_entropy(H, W, t, -100, "mean", 0.0)
    for rank, l, gH, gW, s, e in out:
        assert abs(l - loss) <= 1e-3 * abs(loss)
        assert _maxabs_norm(gH.numpy(), dH[s:e]) <= 2e-2
        assert _maxabs_norm(gW.numpy(), dW) <= 2e-2


@requires_gpu
@two_gpus
def test_vocab_parallel_at_the_cfg5_shard_shape():
    """Vocab-parallel on 2 GPUs with each rank's shard at the size it has in
    the 8-GPU cfg5 run (V_shard = 16032, D = 8192, 65536 rows)."""
    import _dist_gpu_workers as Wk

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    shape = (65536, 8192, 16032 * world)
    procs = [ctx.Process(target=Wk.worker_vocab_shard_check, args=(r, world, port, shape, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=600) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    assert all(o[1] != "error" for o in out), out
    for rank, l, ref, err_h, err_w in out:
        assert abs(l - ref) <= 1e-3 * abs(ref), (l, ref)
        assert err_h <= 2e-2 and err_w <= 2e-2, (err_h, err_w)
