"""World-size-2 Gloo tests of the multi-GPU sharding logic (CPU, no GPU).

Kernels are replaced by CPU stand-ins (tests/_dist_workers.py); the
communication code of greyhound_b200.distributed runs for real. Results are
compared with a single-process computation on the full data."""

import os
import tempfile

import pytest
import torch
import torch.multiprocessing as mp

import _dist_workers as W


def _run(worker, data, world=2, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    fd, store = tempfile.mkstemp(prefix="gh_gloo_")
    os.close(fd)
    os.unlink(store)
    procs = [ctx.Process(target=worker, args=(r, world, store, data, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=timeout) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    return sorted(out, key=lambda x: x[0])


def _data(N=24, D=16, V=40, seed=0, red="mean", z=1e-3):
    g = torch.Generator().manual_seed(seed)
    H = torch.randn(N, D, generator=g)
    Wt = torch.randn(V, D, generator=g) * 0.5
    t = torch.randint(0, V, (N,), generator=g)
    t[::5] = -100
    return H, Wt, t, red, z


def _reference(H, Wt, t, red, z):
    Hr = H.clone().requires_grad_(True)
    Wr = Wt.clone().requires_grad_(True)
    logits = Hr @ Wr.T
    valid = t != -100
    lse = torch.logsumexp(logits, -1)
    ce = torch.nn.functional.cross_entropy(logits, t, ignore_index=-100, reduction="sum")
    loss = ce + z * (lse.square() * valid).sum()
    if red == "mean":
        loss = loss / valid.sum().clamp(min=1)
    loss.backward()
    return loss.item(), Hr.grad, Wr.grad


def test_shard_range_covers_everything():
    from greyhound_b200.distributed import shard_range

    for total in (0, 1, 7, 128256):
        for world in (1, 2, 3, 8):
            spans = [shard_range(total, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            assert max(e - s for s, e in spans) - min(e - s for s, e in spans) <= 1


def test_combine_vocab_stats_is_exact():
    from greyhound_b200.distributed import combine_vocab_stats

    g = torch.Generator().manual_seed(1)
    logits = torch.randn(5, 30, generator=g) * 4
    t = torch.tensor([0, 7, 29, 15, 3])
    parts = []
    for s, e in ((0, 10), (10, 23), (23, 30)):
        lse = torch.logsumexp(logits[:, s:e], -1)
        loc = t - s
        inside = (loc >= 0) & (loc < e - s)
        xt = torch.where(inside, logits[torch.arange(5), t], torch.full((5,), float("-inf")))
        parts.append(torch.stack([lse, torch.ones_like(lse), xt], 1))
    lse, xt = combine_vocab_stats(torch.stack(parts))
    torch.testing.assert_close(lse, torch.logsumexp(logits, -1))
    torch.testing.assert_close(xt, logits[torch.arange(5), t])


@pytest.mark.parametrize("red", ["mean", "sum"])
def test_row_sharded_matches_single_process(red):
    data = _data(red=red)
    out = _run(W.row_sharded_worker, data)
    assert all(o[1] != "error" for o in out), out
    ref_loss, ref_dH, ref_dW = _reference(*data)
    for rank, loss, dH, dW, s, e in out:
        assert abs(loss - ref_loss) <= 1e-5 * max(1, abs(ref_loss))
        torch.testing.assert_close(dH, ref_dH[s:e], rtol=1e-4, atol=1e-5)
        torch.testing.assert_close(dW, ref_dW, rtol=1e-4, atol=1e-5)  # all-reduced on every rank


@pytest.mark.parametrize("red", ["mean", "sum"])
def test_vocab_sharded_matches_single_process(red):
    data = _data(red=red, V=41)
    out = _run(W.vocab_sharded_worker, data)
    assert all(o[1] != "error" for o in out), out
    ref_loss, ref_dH, ref_dW = _reference(*data)
    for rank, loss, dH, dWs, vs, ve in out:
        assert abs(loss - ref_loss) <= 1e-5 * max(1, abs(ref_loss))
        torch.testing.assert_close(dH, ref_dH, rtol=1e-4, atol=1e-5)  # all-reduced partials
        torch.testing.assert_close(dWs, ref_dW[vs:ve], rtol=1e-4, atol=1e-5)


def test_dead_rank_is_detected_not_hung():
    out = _run(W.dead_rank_worker, _data(), timeout=120)
    assert out[1][1] == "left"
    assert out[0][1] == "detected", out


def test_band_exchange_band_arithmetic():
    """Row bands of the fused weight-gradient reduce-scatter: multiples of the
    256-row GEMM tile that cover the vocabulary, every rank owning a
    non-empty band (else the NCCL all-reduce path is taken)."""
    from greyhound_b200.distributed import _band_rows

    for V in (1000, 30011, 32000, 128256, 151936):
        for world in (2, 3, 4, 8):
            b = _band_rows(V, world)
            assert b % 256 == 0 and world * b >= V and b - 256 < -(-V // world)
            last = V - (world - 1) * b
            if last > 0:
                assert last <= b
    assert _band_rows(128256, 8) == 16128
    assert 7 * _band_rows(1000, 8) >= 1000  # too small a vocabulary: no band for the last ranks
