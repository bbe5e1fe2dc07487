"""Workload cfg5 (the Llama-3-70B-scale head: H[65536, 8192], W[128256, 8192]
~ N(0, 0.015), bf16, 2% ignore_index, mean) on one GPU at full size: eight
chunks of 8192 rows (the reference's chunk heuristic,
src/greyhound/ops/chunked_linear_loss.py:24-34) with the weight gradient
accumulated in fp32 across them. Checked against plain fp32 torch of the
reference semantics (bf16 logits, fp32 softmax / CE, fp32 GEMMs): the loss
over all rows, the input gradient on sampled rows and the weight gradient on
sampled vocabulary bands."""

import torch

from greyhound_b200.nn.functional import chunked_linear_cross_entropy
from greyhound_b200.testing import requires_gpu


@requires_gpu
def test_lce_cfg5_full_size_one_gpu():
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(4)
    N, D, V = 65536, 8192, 128256
    H = torch.randn(N, D, device=dev, generator=g).bfloat16()
    W = (torch.randn(V, D, device=dev, generator=g) * 0.015).bfloat16()
    t = torch.randint(0, V, (N,), device=dev, generator=g)
    t[torch.rand(N, device=dev, generator=g) < 0.02] = -100
    Hd = H.clone().requires_grad_(True)
    Wd = W.clone().requires_grad_(True)
    loss = chunked_linear_cross_entropy(Hd, Wd, t)
    loss.backward()
    gH, gW = Hd.grad, Wd.grad
    del Hd, Wd
    torch.cuda.empty_cache()

    valid = t != -100
    n = valid.sum().float()
    rows = torch.arange(0, N, 1021, device=dev)  # sampled rows, every chunk
    bands = [slice(0, 256), slice(64000, 64256), slice(V - 256, V)]  # sampled vocabulary bands
    ref_loss = torch.zeros((), device=dev, dtype=torch.float64)
    lse_all = torch.empty(N, device=dev)
    for s in range(0, N, 4096):
        logits = (H[s:s + 4096] @ W.T).float()  # bf16 logits, as the reference GEMM output
        lse = torch.logsumexp(logits, -1)
        lse_all[s:s + 4096] = lse
        tc = t[s:s + 4096]
        vc = tc != -100
        ref_loss += torch.where(vc, lse - logits.gather(1, tc.clamp(min=0)[:, None])[:, 0], 0.0).double().sum()
        del logits
    ref_loss = (ref_loss / n).item()
    assert abs(loss.item() - ref_loss) <= 1e-3 * abs(ref_loss), (loss.item(), ref_loss)

    def dlogits(r_idx, cols):
        x = (H[r_idx] @ W[cols].T).float()
        p = torch.exp(x - lse_all[r_idx][:, None])
        tt = t[r_idx]
        hit = (tt >= cols.start) & (tt < cols.stop)
        p[hit.nonzero()[:, 0], (tt[hit] - cols.start)] -= 1.0
        p[tt == -100] = 0.0
        return p.bfloat16().float() / n  # the reference's bf16 dlogits, mean scale

    dl = torch.cat([dlogits(rows, slice(v, min(v + 16384, V))) for v in range(0, V, 16384)], dim=1)
    ref_dH = dl @ W.float()
    err = (gH[rows].float() - ref_dH).abs().max() / ref_dH.abs().max()
    assert err <= 2e-2, err.item()
    assert torch.all(gH[~valid] == 0)
    for b in bands:
        ref = torch.zeros(b.stop - b.start, D, device=dev)
        for s in range(0, N, 8192):
            ref += dlogits(torch.arange(s, s + 8192, device=dev), b).T @ H[s:s + 8192].float()
        err = (gW[b].float() - ref).abs().max() / ref.abs().max()
        assert err <= 2e-2, (b, err.item())
