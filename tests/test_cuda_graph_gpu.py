"""The linear cross-entropy step (forward + backward through the public API)
captured in one CUDA graph and replayed: results equal the eager step, and
replay removes the host launch overhead that dominates small shapes (cfg1)."""

import time

import numpy as np
import torch

from greyhound_b200.nn.functional import chunked_linear_cross_entropy
from greyhound_b200.testing import requires_gpu
from oracle import gh_oracle as O


@requires_gpu
def test_lce_step_captures_in_a_cuda_graph():
    dev = torch.device("cuda", 0)
    H, W, t = O.make_lce_inputs(512, 1024, 32000, 0, 0.02, 0.05)  # cfg1
    Hs = torch.from_numpy(H).to(dev, torch.bfloat16).requires_grad_(True)
    Ws = torch.from_numpy(W).to(dev, torch.bfloat16).requires_grad_(True)
    ts = torch.from_numpy(t).to(dev)

    def step():
        Hs.grad = None
        Ws.grad = None
        loss = chunked_linear_cross_entropy(Hs, Ws, ts, z_loss_multiplier=1e-4)
        loss.backward()
        return loss

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(3):  # warm-up outside capture (one-time kernel set-up)
            eager = step()
    torch.cuda.current_stream().wait_stream(s)
    eager_loss = eager.item()
    eager_dH, eager_dW = Hs.grad.clone(), Ws.grad.clone()

    g = torch.cuda.CUDAGraph()
    Hs.grad = None
    Ws.grad = None
    with torch.cuda.graph(g):
        static_loss = chunked_linear_cross_entropy(Hs, Ws, ts, z_loss_multiplier=1e-4)
        static_loss.backward()
    g.replay()
    torch.cuda.synchronize()
    assert static_loss.item() == eager_loss  # deterministic kernels: bit-identical
    assert torch.equal(Hs.grad, eager_dH) and torch.equal(Ws.grad, eager_dW)

    n = 20
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(n):
        g.replay()
    torch.cuda.synchronize()
    t_graph = (time.perf_counter() - t0) / n
    t0 = time.perf_counter()
    for _ in range(n):
        step()
    torch.cuda.synchronize()
    t_eager = (time.perf_counter() - t0) / n
    print(f"cfg1 step: eager {t_eager * 1e3:.3f} ms, graph replay {t_graph * 1e3:.3f} ms")
    assert t_graph <= t_eager * 1.05
