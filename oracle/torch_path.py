"""The reference's own PyTorch path for the linear cross-entropy, on CPU tensors.

TEST AND BASELINE INFRASTRUCTURE ONLY: ``bench.py`` times it on the host
cores as the CPU baseline and as the ``--impl reference`` arm. The product
(``greyhound_b200``) never imports it.

It is the plain-PyTorch computation the reference checks its fused op
against and runs in its forward-only path:

* ``logits = inputs @ weight`` in the activation dtype (bf16), as
  ``reference_linear_cross_entropy`` (src/tests/nn/functional/chunked_linear_loss_test.py:18-42)
  and ``_forward_only_chunked_ce`` (src/greyhound/ops/chunked_linear_cross_entropy.py:91-132);
* ``F.cross_entropy(logits.float(), target, ignore_index=-100, reduction=...)``;
* ``.backward()`` through autograd, which produces ``grad_input`` and
  ``grad_weight`` in bf16 (one dW accumulation per call, as the reference's
  single-chunk case at the Llama-3-8B head shape).
"""

from __future__ import annotations

import time

import torch
import torch.nn.functional as F


def linear_ce_fwd_bwd(inputs: torch.Tensor, weight_dv: torch.Tensor, target: torch.Tensor,
                      reduction: str = "mean", ignore_index: int = -100) -> torch.Tensor:
    """Loss, with ``inputs.grad`` / ``weight_dv.grad`` filled by autograd."""
    logits = inputs @ weight_dv
    loss = F.cross_entropy(logits.float(), target, ignore_index=ignore_index, reduction=reduction)
    loss.backward()
    return loss.detach()


def time_linear_ce(N: int, D: int, V: int, rows: int = 512, repeats: int = 1, seed: int = 2,
                   ignore_frac: float = 0.02, threads: int | None = None) -> dict:
    """Time the reference torch path on one contiguous ``rows``-row slice of
    the ``[N, D] x [D, V]`` workload (bf16, synthetic seeded inputs with the
    workload's distributions). Returns tokens/s and the sample description;
    the first call is a warm-up and is not counted."""
    if threads:
        torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(seed)
    W = (torch.randn(V, D, generator=g) * 0.02).to(torch.bfloat16)
    H = torch.randn(rows, D, generator=g)
    H = (H * torch.rsqrt(H.square().mean(-1, keepdim=True) + 1e-6)).to(torch.bfloat16)
    t = torch.randint(0, V, (rows,), generator=g)
    t[torch.rand(rows, generator=g) < ignore_frac] = -100
    w = W.T.requires_grad_(True)  # [D, V] view, the op's weight convention
    x = H.requires_grad_(True)

    def one():
        x.grad = None
        w.grad = None
        linear_ce_fwd_bwd(x, w, t)

    one()  # warm-up (allocations, oneDNN kernel selection)
    times = []
    for _ in range(repeats):
        t0 = time.perf_counter()
        one()
        times.append(time.perf_counter() - t0)
    best = min(times)
    return {
        "value": rows / best,
        "unit": "tokens/s",
        "cores": torch.get_num_threads(),
        "seconds_per_sample": best,
        "sample": (f"{rows} contiguous rows of the {N}x{D}x{V} workload through the reference torch path "
                   f"(bf16 F.linear, F.cross_entropy on fp32 logits, autograd backward; one dW per sample), "
                   f"best of {repeats} after one warm-up, {best:.2f} s each"),
    }
