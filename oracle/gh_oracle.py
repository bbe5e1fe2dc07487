"""CPU oracle for the greyhound chunked linear cross-entropy hot path (numpy).

TEST INFRASTRUCTURE ONLY. This module is a plain restatement of the
reference algorithm, used as the checker by ``tests/``, by
``__graft_entry__.smoke()`` and as the ``cpu_baseline`` / ``--impl reference``
arm of ``bench.py``. The product (``greyhound_b200``) never imports it and has
no CPU fallback.

Parity of this oracle is pinned by ``tests/test_oracle_golden.py`` against
fixtures in ``tests/golden/`` that were produced by running the reference's
own CPU-runnable code (its test oracles and its forward-only torch path,
see ``tests/golden/make_golden.py``).

Rounding points mirror the reference exactly: the logits GEMM output is
rounded to the activation dtype (bf16) before the CE kernel reads it, the
kernel writes ``dlogits`` in that dtype, ``grad_input`` is produced in that
dtype, ``grad_weight`` is accumulated in fp32 (or the weight dtype) and cast
once, and the mean scaling multiplies the already-rounded gradients.
"""

from __future__ import annotations

import numpy as np

# ---------------------------------------------------------------------------
# bf16 / fp16 emulation


def round_bf16(x: np.ndarray) -> np.ndarray:
    """Round fp32 values to the nearest bf16 (ties to even), returned as fp32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32)
    rounding = ((u >> np.uint32(16)) & np.uint32(1)) + np.uint32(0x7FFF)
    u = (u + rounding) & np.uint32(0xFFFF0000)  # only NaN payloads can wrap; fixed below
    out = u.view(np.float32)
    nan = np.isnan(x)
    if nan.any():
        out = out.copy()
        out[nan] = np.nan
    return out


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round fp32 values to ``dtype`` in {"bf16", "f16", "f32"}; result is fp32."""
    if dtype == "bf16":
        return round_bf16(x)
    if dtype == "f16":
        return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)
    return np.asarray(x, dtype=np.float32)


# ---------------------------------------------------------------------------
# Row kernels


def logsumexp_rows(x: np.ndarray) -> np.ndarray:
    """Per-row natural logsumexp in float64 (the exact value the fp32 kernels approximate)."""
    x = np.asarray(x, dtype=np.float64)
    m = x.max(axis=-1, keepdims=True)
    return (m + np.log(np.exp(x - m).sum(axis=-1, keepdims=True)))[..., 0]


def cross_entropy_with_grad(
    logits: np.ndarray,
    labels: np.ndarray,
    z_loss_multiplier: float,
    ignore_index: int,
    out_dtype: str = "f32",
) -> tuple[float, float, float, np.ndarray]:
    """CE + logits-gradient kernel semantics, src/greyhound/kernels/cross_entropy.py:20-108.

    Per row: ``lse = logsumexp(x)`` (:39-84); for ``label != ignore_index``:
    ``ce += lse - x[label]``, ``z += lse^2``, ``n_valid += 1`` (:85-92);
    gradient ``softmax(x) * (1 + 2 z_mult lse) - onehot(label)``, zero for
    ignored rows (:94-108), rounded to ``out_dtype`` (the logits dtype).
    Returns ``(ce_sum, z_sum, n_valid, dlogits)``.
    """
    x = np.asarray(logits, dtype=np.float64)
    labels = np.asarray(labels, dtype=np.int64)
    rows, V = x.shape
    lse = logsumexp_rows(x)
    valid = labels != ignore_index
    safe = np.where(valid, labels, 0)
    x_lab = x[np.arange(rows), safe]
    ce = float(np.where(valid, lse - x_lab, 0.0).sum())
    z = float(np.where(valid, lse * lse, 0.0).sum())
    n = float(valid.sum())
    p = np.exp(x - lse[:, None])
    g = p * (1.0 + 2.0 * z_loss_multiplier * lse)[:, None]
    g[np.arange(rows), safe] -= valid.astype(np.float64)
    g[~valid] = 0.0
    return ce, z, n, round_to(g.astype(np.float32), out_dtype)


def cross_entropy_loss(
    logits: np.ndarray,
    target: np.ndarray,
    ignore_index: int = -100,
    reduction: str = "mean",
    z_loss_multiplier: float = 0.0,
) -> float:
    """Functional ``cross_entropy`` value (nn/functional.py:72-116; test oracle
    src/tests/nn/functional/cross_entropy_test.py:14-36)."""
    ce, z, n, _ = cross_entropy_with_grad(logits, target, z_loss_multiplier, ignore_index)
    loss = ce + z_loss_multiplier * z
    if reduction == "mean":
        loss /= max(n, 1.0)
    return loss


def selective_log_softmax(logits: np.ndarray, index: np.ndarray) -> np.ndarray:
    """``x[index] - logsumexp(x)`` per row, src/greyhound/kernels/logprobs.py:20-88
    (reduction over the last dim, leading dims flattened, :166-172)."""
    x = np.asarray(logits, dtype=np.float64)
    V = x.shape[-1]
    x2 = x.reshape(-1, V)
    idx = np.asarray(index, dtype=np.int64).reshape(-1)
    lse = logsumexp_rows(x2)
    out = x2[np.arange(x2.shape[0]), idx] - lse
    return out.reshape(np.asarray(index).shape)


def selective_log_softmax_backward(
    logits: np.ndarray, index: np.ndarray, grad_out: np.ndarray
) -> np.ndarray:
    """Gradient of ``sum(grad_out * gather(log_softmax(x), index))`` w.r.t. ``x``.

    The reference has no backward (src/greyhound/ops/logprobs.py:30); this is
    the derivative of its test oracle (src/tests/nn/functional/logprobs_test.py:12-14):
    ``grad_out[r] * (onehot(index[r]) - softmax(x[r]))``.
    """
    x = np.asarray(logits, dtype=np.float64)
    V = x.shape[-1]
    x2 = x.reshape(-1, V)
    idx = np.asarray(index, dtype=np.int64).reshape(-1)
    g = np.asarray(grad_out, dtype=np.float64).reshape(-1)
    lse = logsumexp_rows(x2)
    p = np.exp(x2 - lse[:, None])
    out = -p * g[:, None]
    out[np.arange(x2.shape[0]), idx] += g
    return out.reshape(x.shape).astype(np.float32)


# ---------------------------------------------------------------------------
# Chunked linear cross-entropy

_TARGET_LOGITS_CHUNK_BYTES = 512 * 1024 * 1024
_LARGE_D_MODEL_TARGET_LOGITS_CHUNK_BYTES = 2 * 1024 * 1024 * 1024


def chunk_size(B: int, D: int, V: int, element_size: int) -> int:
    """Rows per chunk, src/greyhound/ops/chunked_linear_loss.py:24-34."""
    base = 1 << (max(-(-B // max(-(-V // D), 1)), 1) - 1).bit_length()
    base = min(max(base, 1), B)
    target = _LARGE_D_MODEL_TARGET_LOGITS_CHUNK_BYTES if D >= 4096 else _TARGET_LOGITS_CHUNK_BYTES
    max_rows = max(target // max(V * element_size, 1), 1)
    memory_limited = min(B, 1 << (max_rows.bit_length() - 1))
    return max(base, memory_limited)


def chunk_step(Hc, W, tc, z_loss_multiplier, ignore_index, dtype, acc, fp32_accum=True):
    """One chunk of the reference loop, src/greyhound/ops/chunked_linear_loss.py:79-101.

    ``logits = round(Hc @ W.T)`` (:82) -> CE + dlogits (:83) -> ``dH = round(dl @ W)``
    (:94) -> ``acc += Hc.T @ dl`` in place (:95-101; rounded to ``dtype`` per
    update when not accumulating in fp32). ``acc`` may be None (forward only).
    Returns ``(ce_sum, z_sum, n_valid, dH_chunk or None)``.
    """
    logits = round_to(Hc @ W.T, dtype)
    ce, z, n, dl = cross_entropy_with_grad(logits, tc, z_loss_multiplier, ignore_index, dtype)
    if acc is None:
        return ce, z, n, None
    dHc = round_to(dl @ W, dtype)
    if fp32_accum:
        acc += Hc.T @ dl
    else:
        acc[...] = round_to(acc + Hc.T @ dl, dtype)
    return ce, z, n, dHc


def chunked_linear_cross_entropy(
    H: np.ndarray,
    W: np.ndarray,
    target: np.ndarray,
    ignore_index: int = -100,
    reduction: str = "mean",
    z_loss_multiplier: float = 0.0,
    fp32_grad_weight_accum: bool = True,
    dtype: str = "bf16",
    chunk: int | None = None,
    with_grad: bool = True,
):
    """Training-path restatement of the reference.

    ``H`` is ``[N, D]``, ``W`` is ``[V, D]`` (values already representable in
    ``dtype``). Follows the chunk loop of
    src/greyhound/ops/chunked_linear_loss.py:56-103 with the CE callback of
    src/greyhound/ops/chunked_linear_cross_entropy.py:43-59, then the mean
    scaling of :159-164. Returns ``(loss, grad_H [N,D], grad_W [V,D])`` (grads
    as fp32 arrays holding ``dtype`` values), or ``loss`` alone when
    ``with_grad`` is False (forward-only path, :91-132).
    """
    H = np.asarray(H, dtype=np.float32)
    W = np.asarray(W, dtype=np.float32)
    target = np.asarray(target, dtype=np.int64)
    N, D = H.shape
    V = W.shape[0]
    elt = 4 if dtype == "f32" else 2
    chunk = chunk or chunk_size(N, D, V, elt)
    ce_sum = z_sum = n_valid = 0.0
    dH = np.zeros((N, D), dtype=np.float32)
    acc = np.zeros((D, V), dtype=np.float32) if with_grad else None
    for s in range(0, N, chunk):
        e = min(s + chunk, N)
        ce, z, n, dHc = chunk_step(H[s:e], W, target[s:e], z_loss_multiplier, ignore_index, dtype,
                                   acc, fp32_grad_weight_accum)
        ce_sum += ce
        z_sum += z
        n_valid += n
        if with_grad:
            dH[s:e] = dHc
    loss = ce_sum + z_loss_multiplier * z_sum
    if reduction == "mean":
        loss /= max(n_valid, 1.0)
    if not with_grad:
        return loss
    dW = round_to(acc, dtype).T.copy()  # cast once (:103), returned as [V, D]
    if reduction == "mean":
        r = np.float32(1.0 / max(n_valid, 1.0))
        dH = round_to(dH * r, dtype)
        dW = round_to(dW * r, dtype)
    return loss, dH, dW


# ---------------------------------------------------------------------------
# Seeded synthetic inputs for the five workload configs (shapes, value
# distributions and ignore fractions as the workload description states).


def _ignore_mask(rng: np.random.Generator, n: int, frac: float) -> np.ndarray:
    k = int(round(frac * n))
    m = np.zeros(n, dtype=bool)
    m[rng.choice(n, size=k, replace=False)] = True
    return m


def make_lce_inputs(N: int, D: int, V: int, seed: int, w_std: float, ignore_frac: float,
                    rms_norm: bool = False, ignore_index: int = -100):
    """``H ~ N(0,1)`` (optionally RMS-normalised per row), ``W ~ N(0, w_std)``,
    uniform targets with ``ignore_frac`` set to ``ignore_index``; bf16 values."""
    rng = np.random.default_rng(seed)
    H = rng.standard_normal((N, D), dtype=np.float32)
    if rms_norm:
        H = H / np.sqrt((H * H).mean(axis=1, keepdims=True) + 1e-6)
    W = rng.standard_normal((V, D), dtype=np.float32) * np.float32(w_std)
    t = rng.integers(0, V, size=N, dtype=np.int64)
    t[_ignore_mask(rng, N, ignore_frac)] = ignore_index
    return round_bf16(H), round_bf16(W), t


def make_ce_inputs(rows: int, V: int, seed: int, std: float = 2.0, spike: float = 8.0,
                   spike_frac: float = 0.01, ignore_frac: float = 0.03, ignore_index: int = -100):
    """Logits ``N(0, std)`` plus ``+spike`` on a random ``spike_frac`` of each row's
    entries; labels uniform with ``ignore_frac`` ignored; bf16 values."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((rows, V), dtype=np.float32) * np.float32(std)
    k = max(1, int(spike_frac * V))
    cols = rng.integers(0, V, size=(rows, k))
    x[np.arange(rows)[:, None], cols] += np.float32(spike)
    t = rng.integers(0, V, size=rows, dtype=np.int64)
    t[_ignore_mask(rng, rows, ignore_frac)] = ignore_index
    return round_bf16(x), t


def make_sls_inputs(rows: int, V: int, seed: int, std: float = 3.0):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((rows, V), dtype=np.float32) * np.float32(std)
    idx = rng.integers(0, V, size=rows, dtype=np.int64)
    return round_bf16(x), idx
