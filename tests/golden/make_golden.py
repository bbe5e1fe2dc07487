"""Generate the golden fixtures in tests/golden/ from the reference's own code.

Run in a container where the reference checkout is importable (its CPU-only
paths: the pure-torch test oracles, the forward-only chunked CE and the
generic chunk loop); the fixtures are committed so that tests never need the
reference at run time:

    python tests/golden/make_golden.py --reference-src <greyhound>/src

Inputs come from the seeded generators in ``oracle/gh_oracle.py`` (numpy,
deterministic), so large inputs are not stored: tests regenerate them from
the seed and compare against the stored outputs.
"""

from __future__ import annotations

import argparse
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from oracle import gh_oracle as O  # noqa: E402


def _bf16(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(torch.bfloat16)


def gen_ce(ref_ce) -> dict:
    """Standalone CE: the reference test oracle (cross_entropy_test.py:14-36) + autograd."""
    out = {}
    cases = [("ce37x257", 37, 257, 11), ("ce16x257", 16, 257, 12), ("ce64x4099", 64, 4099, 13)]
    for name, rows, V, seed in cases:
        x, t = O.make_ce_inputs(rows, V, seed, ignore_frac=0.2)
        small = rows * V <= 1 << 14
        if small:
            out[f"{name}/logits"] = x
            out[f"{name}/target"] = t
        sel = np.random.default_rng(seed + 200).integers(0, x.size, size=4096)
        for red in ("sum", "mean"):
            for z in (0.0, 1e-4):
                xt = torch.from_numpy(x).requires_grad_(True)
                loss = ref_ce(xt, torch.from_numpy(t), reduction=red, z_loss_multiplier=z)
                loss.backward()
                out[f"{name}/{red}/z{z}/loss"] = np.float64(loss.item())
                g = xt.grad.numpy().astype(np.float32)
                if small:
                    out[f"{name}/{red}/z{z}/grad"] = g
                else:
                    out[f"{name}/{red}/z{z}/grad_sel"] = sel
                    out[f"{name}/{red}/z{z}/grad_vals"] = g.reshape(-1)[sel]
    return out


def gen_sls(ref_sls) -> dict:
    """Selective log-softmax: the reference test oracle (logprobs_test.py:12-14) + autograd."""
    out = {}
    for name, shape, seed in (("sls4x16x257", (4, 16, 257), 21), ("sls8x513", (8, 513), 22),
                              ("sls16x151936", (16, 151936), 23)):
        rows = int(np.prod(shape[:-1]))
        x, idx = O.make_sls_inputs(rows, shape[-1], seed)
        x = x.reshape(shape)
        idx = idx.reshape(shape[:-1])
        g = np.random.default_rng(seed + 100).standard_normal(idx.shape).astype(np.float32)
        xt = torch.from_numpy(x).requires_grad_(True)
        res = ref_sls(xt, torch.from_numpy(idx))
        (res * torch.from_numpy(g)).sum().backward()
        out[f"{name}/out"] = res.detach().numpy().astype(np.float32)
        out[f"{name}/grad_out"] = g
        if rows * shape[-1] <= 1 << 16:
            out[f"{name}/logits"] = x
            out[f"{name}/index"] = idx
            out[f"{name}/grad"] = xt.grad.numpy().astype(np.float32)
        else:
            # large case: store a seeded subset of the gradient
            sel = np.random.default_rng(seed + 200).integers(0, x.size, size=4096)
            out[f"{name}/grad_sel"] = sel
            out[f"{name}/grad_vals"] = xt.grad.numpy().reshape(-1)[sel].astype(np.float32)
    return out


class _CpuAddmm:
    """``torch.addmm(..., out_dtype=...)`` exists only for CUDA. On the CPU the
    reference loop's fp32-accumulated weight-gradient update
    (ops/chunked_linear_loss.py:95-101) is evaluated as the same product of
    bf16 values accumulated in fp32."""

    def __init__(self):
        self.orig = torch.addmm

    def __call__(self, input, mat1, mat2, *, out=None, out_dtype=None, **kw):
        if out_dtype is None:
            return self.orig(input, mat1, mat2, out=out, **kw)
        res = (input.float() + mat1.float() @ mat2.float()).to(out_dtype)
        if out is not None:
            out.copy_(res)
            return out
        return res

    def __enter__(self):
        torch.addmm = self
        return self

    def __exit__(self, *a):
        torch.addmm = self.orig


def gen_lce(ref_lce, fwd_only, loop, chunk_fn) -> dict:
    """Linear CE: the reference test oracle (chunked_linear_loss_test.py:18-42), the
    reference forward-only torch path (ops/chunked_linear_cross_entropy.py:91-132)
    and the reference chunk loop (ops/chunked_linear_loss.py:56-103) driven by a
    torch CE callback with the kernel's semantics."""
    out = {}

    def ce_callback(target, z, ignore):
        def cb(logits_chunk, s, e):
            lg = logits_chunk.detach().float().requires_grad_(True)
            t = target[s:e]
            loss = torch.nn.functional.cross_entropy(lg, t, ignore_index=ignore, reduction="sum")
            if z > 0:
                valid = t != ignore
                loss = loss + z * (torch.logsumexp(lg, -1).square() * valid).sum()
            (g,) = torch.autograd.grad(loss, lg)
            return loss.detach(), g.to(logits_chunk.dtype)

        return cb

    cases = [
        # name, N, D, V, seed, w_std, ignore_frac, rms, chunk
        ("lce32x128x1000", 32, 128, 1000, 31, 1.0, 0.25, False, None),
        ("lce37x64x257c11", 37, 64, 257, 32, 1.0, 0.2, False, 11),
        ("cfg1", 512, 1024, 32000, 0, 0.02, 0.05, False, None),
    ]
    for name, N, D, V, seed, w_std, ign, rms, chunk in cases:
        H, W, t = O.make_lce_inputs(N, D, V, seed, w_std, ign, rms_norm=rms)
        Ht, Wt, tt = _bf16(H), _bf16(W), torch.from_numpy(t)
        small = N * D + V * D <= 1 << 18
        if small:
            out[f"{name}/H"] = H
            out[f"{name}/W"] = W
            out[f"{name}/target"] = t
        for red in ("mean", "sum"):
            for z in (0.0, 1e-4):
                key = f"{name}/{red}/z{z}"
                # forward-only reference path: bf16 GEMM, fp32 CE
                out[f"{key}/loss_fwd_only"] = np.float64(
                    fwd_only(Ht, Wt.T, tt, -100, red, z).item()
                )
                # reference chunk loop with the CE-kernel-semantics callback
                with _CpuAddmm():
                    loss_sum, gH, gW = loop(Ht, Wt.T, ce_callback(tt, z, -100), True, chunk)
                n_valid = float((t != -100).sum())
                if red == "mean":
                    r = torch.tensor(1.0 / max(n_valid, 1.0))
                    loss = loss_sum / max(n_valid, 1.0)
                    gH = gH.mul_(r)
                    gW = gW.mul_(r)
                else:
                    loss = loss_sum
                out[f"{key}/loss"] = np.float64(loss.item())
                gH = gH.float().numpy()
                gW = gW.float().numpy().T  # [V, D]
                if small:
                    out[f"{key}/grad_H"] = gH
                    out[f"{key}/grad_W"] = gW
                else:
                    rng = np.random.default_rng(seed + 300)
                    sh = rng.integers(0, gH.size, size=4096)
                    sw = rng.integers(0, gW.size, size=4096)
                    out[f"{key}/grad_H_sel"] = sh
                    out[f"{key}/grad_H_vals"] = gH.reshape(-1)[sh]
                    out[f"{key}/grad_W_sel"] = sw
                    out[f"{key}/grad_W_vals"] = gW.reshape(-1)[sw]
                    out[f"{key}/grad_H_sumsq"] = np.float64((gH.astype(np.float64) ** 2).sum())
                    out[f"{key}/grad_W_sumsq"] = np.float64((gW.astype(np.float64) ** 2).sum())
                if small and red == "mean":
                    # the reference *test oracle* (fp32 autograd through the bf16 GEMM)
                    Hr = Ht.clone().requires_grad_(True)
                    Wr = Wt.clone().requires_grad_(True)
                    lr = ref_lce(Hr, Wr.T, tt, reduction=red, z_loss_multiplier=z)
                    lr.backward()
                    out[f"{key}/test_oracle_loss"] = np.float64(lr.item())
                    out[f"{key}/test_oracle_grad_H"] = Hr.grad.float().numpy()
                    out[f"{key}/test_oracle_grad_W"] = Wr.grad.float().numpy()
            if name == "cfg1":
                break  # one reduction is enough for the large CPU case
    table = []
    for B, D, V, elt in [(512, 1024, 32000, 2), (8192, 4096, 128256, 2), (65536, 8192, 128256, 2),
                         (8192, 8192, 16032, 2), (65536, 8192, 16032, 2), (32, 128, 1000, 2),
                         (37, 64, 257, 2), (16, 64, 256, 4), (1024, 2048, 151936, 2), (1, 8, 3, 2)]:
        table.append((B, D, V, elt, chunk_fn(B, D, V, elt)))
    out["chunk_table"] = np.array(table, dtype=np.int64)
    return out


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-src", required=True)
    ap.add_argument("--out", default=str(HERE / "golden.npz"))
    args = ap.parse_args()
    sys.path.insert(0, args.reference_src)
    from greyhound.ops.chunked_linear_cross_entropy import _forward_only_chunked_ce
    from greyhound.ops.chunked_linear_loss import (
        _chunked_linear_loss_chunk_size,
        _chunked_linear_loss_with_grad,
    )
    from tests.nn.functional.chunked_linear_loss_test import reference_linear_cross_entropy
    from tests.nn.functional.cross_entropy_test import reference_cross_entropy
    from tests.nn.functional.logprobs_test import reference_selective_log_softmax

    torch.set_num_threads(max(1, torch.get_num_threads()))
    data = {}
    data.update(gen_ce(reference_cross_entropy))
    data.update(gen_sls(reference_selective_log_softmax))
    data.update(
        gen_lce(
            reference_linear_cross_entropy,
            _forward_only_chunked_ce,
            _chunked_linear_loss_with_grad,
            _chunked_linear_loss_chunk_size,
        )
    )
    np.savez_compressed(args.out, **data)
    print(f"wrote {args.out}: {len(data)} arrays, {Path(args.out).stat().st_size / 1e3:.0f} kB")
    return 0


if __name__ == "__main__":
    sys.exit(main())
