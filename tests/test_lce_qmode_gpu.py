"""The bf16 linear-CE pipeline without a logits -> dlogits pass.

The logits GEMM stores q = e^x (bf16) in place of the logits; one value per
row (the target column) is then rewritten so that the row times a per-row
factor alpha is the reference's logits gradient; the weight-gradient GEMM
reads q with H scaled by alpha, and the input-gradient GEMM applies alpha in
its epilogue. Rows with a group whose largest logit falls outside e^x's safe
exponent window store raw logits and are rewritten by a fix-up pass. These
tests drive every branch against the oracle (the reference's chunk loop,
src/greyhound/ops/chunked_linear_loss.py:56-103) and against the previous
pipeline (logits written, then rewritten in place)."""

import os

import numpy as np
import pytest
import torch

from greyhound_b200.nn.functional import chunked_linear_cross_entropy
from greyhound_b200.testing import requires_gpu
from oracle import gh_oracle as O


def _maxabs_norm(a, ref):
    a = np.asarray(a, np.float64)
    ref = np.asarray(ref, np.float64)
    return np.abs(a - ref).max() / max(np.abs(ref).max(), 1e-30)


def _run(H, W, t, red="mean", z=1e-4, accum="fp32"):
    dev = torch.device("cuda", 0)
    Hd = torch.from_numpy(H).to(dev, torch.bfloat16).requires_grad_(True)
    Wd = torch.from_numpy(W).to(dev, torch.bfloat16).requires_grad_(True)
    loss = chunked_linear_cross_entropy(Hd, Wd, torch.from_numpy(t).to(dev), reduction=red,
                                        z_loss_multiplier=z, grad_weight_accum_dtype=accum)
    loss.backward()
    return loss.item(), Hd.grad.float().cpu().numpy(), Wd.grad.float().cpu().numpy()


def _check(H, W, t, red="mean", z=1e-4, accum="fp32"):
    loss, gH, gW = _run(H, W, t, red, z, accum)
    oloss, odH, odW = O.chunked_linear_cross_entropy(H, W, t, -100, red, z, fp32_grad_weight_accum=accum == "fp32")
    assert np.isfinite(loss) and np.all(np.isfinite(gH)) and np.all(np.isfinite(gW))
    assert abs(loss - oloss) <= 1e-3 * max(1.0, abs(oloss)), (loss, oloss)
    assert _maxabs_norm(gH, odH) <= 2e-2
    assert _maxabs_norm(gW, odW) <= 2e-2
    assert np.all(gH[t == -100] == 0)


def _inputs(N, D, V, seed, w_std, ign=0.1):
    return O.make_lce_inputs(N, D, V, seed, w_std, ign)


@requires_gpu
@pytest.mark.parametrize("red", ["mean", "sum"])
def test_large_logits_take_the_fixup_path(red):
    # logits with a standard deviation of ~34: every row group's maximum is
    # far above the e^x window, so all rows are stored raw and normalised
    H, W, t = _inputs(96, 128, 3000, 41, 3.0)
    _check(H, W, t, red)


@requires_gpu
def test_mixed_rows_in_and_out_of_the_window():
    H, W, t = _inputs(300, 128, 5000, 42, 1.0)
    H[::3] = O.round_bf16(H[::3] * 6.0)  # every third row far outside the window
    _check(H, W, t)


def _exact(H, W, t, z):
    """Float64 gradients of the mean loss from the bf16-rounded logits, no
    other rounding: the yardstick when bf16 rounding noise dominates."""
    x = O.round_bf16(H @ W.T).astype(np.float64)
    m = x.max(1, keepdims=True)
    e = np.exp(x - m)
    lse = (m + np.log(e.sum(1, keepdims=True)))
    p = e / e.sum(1, keepdims=True)
    valid = t != -100
    g = p * (1 + 2 * z * lse)
    g[np.arange(len(t))[valid], t[valid]] -= 1.0
    g[~valid] = 0
    g /= max(valid.sum(), 1)
    return g @ W.astype(np.float64), g.T @ H.astype(np.float64)


@requires_gpu
def test_very_negative_logits():
    # column 0 shifts every logit of the first half of the rows by about -128;
    # dH[:, 0] is then a cancellation of terms 8x larger than the result, so
    # both this path and the reference's bf16 dlogits carry rounding noise of
    # that size: compare each against the exact gradient
    H, W, t = _inputs(128, 64, 2000, 43, 0.1)
    W[:, 0] = -8.0
    H[:64, 0] = 16.0
    z = 1e-4
    loss, gH, gW = _run(H, W, t, "mean", z)
    oloss, odH, odW = O.chunked_linear_cross_entropy(H, W, t, -100, "mean", z)
    assert abs(loss - oloss) <= 1e-3 * max(1.0, abs(oloss))
    eH, eW = _exact(H, W, t, z)
    for got, ref, ex in ((gH, odH, eH), (gW, odW, eW)):
        err, ref_err = np.abs(got - ex).max(), np.abs(ref - ex).max()
        assert err <= max(2.0 * ref_err, 2e-2 * np.abs(ex).max()), (err, ref_err)


@requires_gpu
@pytest.mark.parametrize("gain", [0.08, 0.12])
def test_confident_predictions_keep_their_precision(gain):
    # W[t_r] aligned with H_r: the target probability is 0.9 (gain 0.08) or
    # 0.9996 (gain 0.12), so the gradient at the target is a small difference
    # p_t - 1 that must not be formed from rounded values
    H, W, t = _inputs(512, 128, 2000, 47, 0.02, ign=0.0)
    t[:] = np.arange(512)
    W[:512] = O.round_bf16(H[:512] * gain)
    _check(H, W, t)


@requires_gpu
def test_repeated_targets_are_summed_once_each():
    H, W, t = _inputs(512, 128, 4000, 44, 0.1, ign=0.0)
    t[::2] = 7
    t[1::4] = 123
    t[3::8] = -100
    _check(H, W, t)
    _check(H, W, t, accum="weight")


@requires_gpu
def test_multi_chunk_weight_accumulation():
    # 2 GiB / (V * 2 B) rows per chunk would be one chunk; a small D gives
    # several chunks through the reference heuristic (D < 4096: 512 MiB)
    H, W, t = _inputs(4096, 256, 131072 + 37, 45, 0.05, ign=0.05)
    _check(H, W, t)


@requires_gpu
def test_q_store_matches_the_dlogits_pipeline(monkeypatch):
    H, W, t = _inputs(1024, 512, 32000, 46, 0.05, ign=0.05)
    q = _run(H, W, t)
    monkeypatch.setenv("GREYHOUND_B200_LCE_Q", "0")
    assert os.environ["GREYHOUND_B200_LCE_Q"] == "0"
    ref = _run(H, W, t)
    assert abs(q[0] - ref[0]) <= 1e-5 * abs(ref[0])
    assert _maxabs_norm(q[1], ref[1]) <= 1e-2
    assert _maxabs_norm(q[2], ref[2]) <= 1e-2


@requires_gpu
def test_gradients_in_backward_follow_grad_output(monkeypatch):
    """Single-chunk calls compute both gradients in the backward, multiplied
    by grad_output in the GEMM epilogues: a retained graph's second backward
    with another grad_output gives that multiple, and the results match the
    gradients-in-forward schedule (GREYHOUND_B200_LCE_TWO_PHASE=0)."""
    H, W, t = _inputs(512, 256, 8000, 48, 0.05, ign=0.05)
    dev = torch.device("cuda", 0)
    Hd = torch.from_numpy(H).to(dev, torch.bfloat16).requires_grad_(True)
    Wd = torch.from_numpy(W).to(dev, torch.bfloat16).requires_grad_(True)
    loss = chunked_linear_cross_entropy(Hd, Wd, torch.from_numpy(t).to(dev), z_loss_multiplier=1e-4)
    loss.backward(retain_graph=True)
    g1 = (Hd.grad.float().clone(), Wd.grad.float().clone())
    Hd.grad = None
    Wd.grad = None
    loss.backward(torch.tensor(2.5, device=dev))
    for a, b in zip((Hd.grad.float(), Wd.grad.float()), g1):
        assert (a - 2.5 * b).abs().max() <= 1e-2 * (2.5 * b).abs().max()
    monkeypatch.setenv("GREYHOUND_B200_LCE_TWO_PHASE", "0")
    ref = _run(H, W, t, "mean", 1e-4)
    assert abs(loss.item() - ref[0]) <= 1e-5 * abs(ref[0])
    assert _maxabs_norm(g1[0].cpu().numpy(), ref[1]) <= 1e-2
    assert _maxabs_norm(g1[1].cpu().numpy(), ref[2]) <= 1e-2
