"""Chunked linear cross-entropy forward+backward on the device.

Computes, for ``logits = inputs @ weight`` (``weight`` given as the ``[D, V]``
view the ops layer passes, src/greyhound/nn/functional.py:279):
``ce_sum``, ``z_sum``, ``n_valid``, ``grad_input = dlogits @ weight.T`` and
``grad_weight = inputs.T @ dlogits`` with
``dlogits = softmax(logits) * (1 + 2 z lse) - onehot(target)`` (0 on ignored rows),
following the chunk loop of src/greyhound/ops/chunked_linear_loss.py:56-103 and the
callback of src/greyhound/ops/chunked_linear_cross_entropy.py:43-59.
"""

from __future__ import annotations

import os

import torch
from torch import Tensor

from greyhound_b200.kernels.cross_entropy import cross_entropy_with_grad

# SMs left free for a collective that overlaps the deferred dH GEMM
# (GREYHOUND_B200_COMM_SMS overrides).
_COMM_SMS = 32

__all__ = ["linear_cross_entropy_with_grad", "linear_cross_entropy_loss", "chunk_size_for"]

_TARGET_LOGITS_CHUNK_BYTES = 512 * 1024 * 1024
_LARGE_D_MODEL_TARGET_LOGITS_CHUNK_BYTES = 2 * 1024 * 1024 * 1024


def _next_power_of_2(n: int) -> int:
    return 1 << (n - 1).bit_length()


def _prev_power_of_2(n: int) -> int:
    return 1 << (n.bit_length() - 1)


def chunk_size_for(B: int, D: int, V: int, element_size: int) -> int:
    """Rows per logits chunk: the reference heuristic, ops/chunked_linear_loss.py:24-34.

    ``max(next_pow2(ceil(B / ceil(V / D))), min(B, prev_pow2(T // (V * elt))))``
    with ``T`` = 2 GiB when ``D >= 4096`` else 512 MiB.
    """
    base = _next_power_of_2(-(-B // max(-(-V // D), 1)))
    base = min(max(base, 1), B)
    target = _LARGE_D_MODEL_TARGET_LOGITS_CHUNK_BYTES if D >= 4096 else _TARGET_LOGITS_CHUNK_BYTES
    max_rows = max(target // max(V * element_size, 1), 1)
    return max(base, min(B, _prev_power_of_2(max_rows)))


def _check(inputs: Tensor, weight: Tensor, target: Tensor) -> None:
    if inputs.ndim != 2 or weight.ndim != 2 or inputs.shape[1] != weight.shape[0]:
        raise ValueError(
            f"expected inputs [B, D] and weight [D, V], got {tuple(inputs.shape)} and {tuple(weight.shape)}"
        )
    if target.shape != (inputs.shape[0],):
        raise ValueError(f"expected target shape {(inputs.shape[0],)}, got {tuple(target.shape)}")
    if not inputs.is_cuda or weight.device != inputs.device or target.device != inputs.device:
        raise ValueError("expected inputs, weight and target on the same CUDA device")


def _tc_ok(inputs: Tensor, weight: Tensor) -> bool:
    """bf16/fp16 with a hidden size that gives 16-byte rows -> tcgen05 pipeline.
    fp32 (the reference's opcheck dtype) stays on cuBLAS GEMMs + the row kernel."""
    return (
        inputs.dtype in (torch.bfloat16, torch.float16)
        and weight.dtype == inputs.dtype
        and inputs.shape[1] % 8 == 0
    )


def _weight_vd(weight: Tensor) -> Tensor:
    """The [V, D] row-major matrix behind the [D, V] operand (a view when it is W.T)."""
    w = weight.T
    return w if w.is_contiguous() else w.contiguous()


def _tc_lce(inputs, weight, target, z, fp32_accum, ignore_index, mean, grad_scale, with_grad,
            grad_weight_hook=None):
    from greyhound_b200 import _lib

    B, D = inputs.shape
    V = weight.shape[1]
    x = inputs.contiguous()
    w = _weight_vd(weight)
    t = target.contiguous()
    dev = inputs.device
    chunk = chunk_size_for(B, D, V, inputs.element_size())
    lib = _lib.load()
    _lib.raise_pending(dev, "linear_cross_entropy")
    code = _lib.dtype_code(inputs.dtype)
    if with_grad:
        ws_bytes = lib.gh_lce_workspace_bytes(B, D, V, chunk, code, int(fp32_accum))
    else:  # statistics only: the logits never touch memory
        ws_bytes = lib.gh_lce_loss_workspace_bytes(B, D, V, chunk, code)
    ws = _lib.workspace(ws_bytes, dev)
    ce_sum = torch.empty((), dtype=torch.float32, device=dev)
    z_sum = torch.empty((), dtype=torch.float32, device=dev)
    n_valid = torch.empty((), dtype=torch.float32, device=dev)
    gi = torch.empty((B, D), dtype=inputs.dtype, device=dev) if with_grad else None
    # [V, D] row-major; returned as the [D, V] view (see _fake in the ops layer)
    gw = torch.empty((V, D), dtype=weight.dtype, device=dev) if with_grad else None
    gs = grad_scale.reshape(1).float().contiguous() if grad_scale is not None else None
    defer = with_grad and grad_weight_hook is not None and B > 0
    stream = _lib.stream_of(inputs)
    st = lib.gh_lce_fwd_bwd(
        x.data_ptr(), w.data_ptr(), t.data_ptr(), B, D, V, code, float(z), int(ignore_index),
        int(mean), _lib.ptr(gs), chunk, int(fp32_accum),
        _lib.GH_LCE_DEFER_LAST_DH if defer else 0,
        _lib.ptr(gi), _lib.ptr(gw), ce_sum.data_ptr(), z_sum.data_ptr(), n_valid.data_ptr(),
        ws.data_ptr(), ws.numel(), stream,
    )
    _lib.check(st, "linear_cross_entropy")
    _lib.raise_on_status(ws, "linear_cross_entropy")
    if defer:
        work = grad_weight_hook(gw)
        # The last chunk's dH runs in two parts: the first on fewer SMs, so the
        # collective's kernels (NVLS all-reduce: 24 CTAs) can run beside it, the
        # second on all SMs once the collective is done (stream-ordered by
        # work.wait()). Measured at 2 GPUs: 32 reserved SMs 21.6 ms/step, 24:
        # 21.9, 0 (one full-grid launch): 22.7.
        sms = torch.cuda.get_device_properties(dev).multi_processor_count
        reserve = int(os.environ.get("GREYHOUND_B200_COMM_SMS", str(_COMM_SMS)))
        last_rows = B - ((B - 1) // chunk) * chunk
        if work is None or reserve > 0:
            # first part on fewer SMs beside the collective, rest on all SMs after it
            split = min((last_rows // 2 + 255) // 256 * 256, last_rows) if work is not None else last_rows
            ctas = max(2, sms - reserve) if work is not None else 0
        else:
            split, ctas = last_rows, 0  # whole dH on all SMs, overlapping the collective
        st = lib.gh_lce_dh_last_chunk(
            w.data_ptr(), B, D, V, code, chunk, int(fp32_accum), 0, split, None, gi.data_ptr(), ws.data_ptr(),
            ws.numel(), ctas, stream,
        )
        _lib.check(st, "linear_cross_entropy dH")
        if work is not None:
            work.wait()
        st = lib.gh_lce_dh_last_chunk(
            w.data_ptr(), B, D, V, code, chunk, int(fp32_accum), split, -1, None, gi.data_ptr(), ws.data_ptr(),
            ws.numel(), 0, stream,
        )
        _lib.check(st, "linear_cross_entropy dH")
    elif with_grad and grad_weight_hook is not None:
        w_ = grad_weight_hook(gw)
        if w_ is not None:
            w_.wait()
    return ce_sum, z_sum, n_valid, gi, (gw.T if gw is not None else None)


def linear_cross_entropy_with_grad(
    inputs: Tensor,
    weight: Tensor,
    target: Tensor,
    z_loss_multiplier: float,
    fp32_grad_weight_accum: bool,
    ignore_index: int,
    mean_reduction: bool = False,
    grad_scale: Tensor | None = None,
    grad_weight_hook=None,
) -> tuple[Tensor, Tensor, Tensor, Tensor, Tensor]:
    """Returns ``(ce_sum, z_sum, n_valid, grad_input [B, D], grad_weight [D, V])``.

    ``grad_weight`` is the transposed view of a row-major ``[V, D]`` tensor:
    the layout of ``W.grad`` for the ``[V, D]`` parameter the functional API
    takes, so autograd accumulates it without a re-layout copy.

    With ``mean_reduction`` both gradients are already divided by
    ``max(n_valid, 1)``; ``grad_scale`` (1-element fp32 device tensor)
    multiplies them further. ``grad_weight_hook(grad_weight)`` runs as soon as
    the final weight gradient exists (the data-parallel all-reduce hooks in here).
    """
    _check(inputs, weight, target)
    if _tc_ok(inputs, weight):
        return _tc_lce(inputs, weight, target, z_loss_multiplier, fp32_grad_weight_accum, ignore_index,
                       mean_reduction, grad_scale, True, grad_weight_hook)
    # fp32 operands: the CE row kernel between fp32 GEMMs emulated on the
    # bf16 tcgen05 GEMM (kernels/gemm.py:gemm_nt_fp32)
    from greyhound_b200.kernels.gemm import gemm_nt_fp32

    B, D = inputs.shape
    V = weight.shape[1]
    chunk = chunk_size_for(B, D, V, inputs.element_size())
    dev = inputs.device
    target = target.contiguous()
    ce_sum = torch.zeros((), dtype=torch.float32, device=dev)
    z_sum = torch.zeros((), dtype=torch.float32, device=dev)
    n_valid = torch.zeros((), dtype=torch.float32, device=dev)
    grad_input = torch.empty_like(inputs)
    acc_dtype = torch.float32 if fp32_grad_weight_accum else weight.dtype
    grad_weight_acc = torch.zeros((V, D), dtype=acc_dtype, device=dev)
    scale = grad_scale.reshape(1).float() if grad_scale is not None else None
    if mean_reduction:
        m = 1.0 / (target != ignore_index).sum().float().clamp(min=1.0).reshape(1)
        scale = m if scale is None else scale * m
    for s in range(0, B, chunk):
        e = min(s + chunk, B)
        x = inputs[s:e]
        logits = gemm_nt_fp32(x, weight.T).to(inputs.dtype)
        c, z, n = cross_entropy_with_grad(
            logits, target[s:e], z_loss_multiplier, ignore_index, logits, grad_scale=scale
        )
        ce_sum += c
        z_sum += z
        n_valid += n
        grad_input[s:e] = gemm_nt_fp32(logits, weight).to(inputs.dtype)
        if acc_dtype == torch.float32:
            gemm_nt_fp32(logits.T, x.T, out=grad_weight_acc, addend=grad_weight_acc)
        else:
            grad_weight_acc += gemm_nt_fp32(logits.T, x.T).to(acc_dtype)
    grad_weight_vd = grad_weight_acc.to(weight.dtype)
    if grad_weight_hook is not None:
        work = grad_weight_hook(grad_weight_vd)
        if work is not None:
            work.wait()
    grad_weight = grad_weight_vd.T
    return ce_sum, z_sum, n_valid, grad_input, grad_weight


def two_phase_ok(inputs: Tensor, weight: Tensor) -> bool:
    """Whether the loss / gradient split applies (gradients computed in the
    backward, already scaled by grad_output): tcgen05 operands and all rows
    in one chunk (the Llama-3-8B head's case). GREYHOUND_B200_LCE_TWO_PHASE=0
    keeps the reference's gradients-in-forward schedule."""
    if os.environ.get("GREYHOUND_B200_LCE_TWO_PHASE", "1") in ("0", ""):
        return False
    if inputs.ndim != 2 or weight.ndim != 2 or not inputs.is_cuda or not _tc_ok(inputs, weight):
        return False
    B, D = inputs.shape
    V = weight.shape[1]
    return B > 0 and chunk_size_for(B, D, V, inputs.element_size()) >= B


def lce_workspace_bytes(inputs: Tensor, weight: Tensor, fp32_accum: bool) -> int:
    from greyhound_b200 import _lib

    B, D = inputs.shape
    V = weight.shape[1]
    chunk = chunk_size_for(B, D, V, inputs.element_size())
    return max(int(_lib.load().gh_lce_workspace_bytes(B, D, V, chunk, _lib.dtype_code(inputs.dtype),
                                                       int(fp32_accum))), 256)


def linear_cross_entropy_stats_keep(inputs: Tensor, weight: Tensor, target: Tensor, z_loss_multiplier: float,
                                    fp32_accum: bool, ignore_index: int, mean_reduction: bool,
                                    grad_scale: Tensor | None = None) -> tuple[Tensor, Tensor, Tensor, Tensor]:
    """Phase 1 of the split: ``(ce_sum, z_sum, n_valid, workspace)``. The
    workspace keeps what both gradient GEMMs need (the stored e^x tile and
    the per-row factors, with the mean / grad_scale folded in) for
    ``linear_cross_entropy_grads_from``."""
    from greyhound_b200 import _lib

    _check(inputs, weight, target)
    B, D = inputs.shape
    V = weight.shape[1]
    x = inputs.contiguous()
    w = _weight_vd(weight)
    t = target.contiguous()
    dev = inputs.device
    lib = _lib.load()
    _lib.raise_pending(dev, "linear_cross_entropy")
    chunk = chunk_size_for(B, D, V, inputs.element_size())
    ws = _lib.workspace(lce_workspace_bytes(inputs, weight, fp32_accum), dev)
    ce_sum = torch.empty((), dtype=torch.float32, device=dev)
    z_sum = torch.empty((), dtype=torch.float32, device=dev)
    n_valid = torch.empty((), dtype=torch.float32, device=dev)
    gs = grad_scale.reshape(1).float().contiguous() if grad_scale is not None else None
    st = lib.gh_lce_fwd_bwd(
        x.data_ptr(), w.data_ptr(), t.data_ptr(), B, D, V, _lib.dtype_code(inputs.dtype), float(z_loss_multiplier),
        int(ignore_index), int(mean_reduction), _lib.ptr(gs), chunk, int(fp32_accum), _lib.GH_LCE_GRADS_LATER,
        None, None, ce_sum.data_ptr(), z_sum.data_ptr(), n_valid.data_ptr(), ws.data_ptr(), ws.numel(),
        _lib.stream_of(x))
    _lib.check(st, "linear_cross_entropy")
    _lib.raise_on_status(ws, "linear_cross_entropy")
    return ce_sum, z_sum, n_valid, ws


def linear_cross_entropy_grads_from(ws: Tensor, inputs: Tensor, weight: Tensor, fp32_accum: bool,
                                    grad_output: Tensor | None) -> tuple[Tensor, Tensor]:
    """Phase 2: ``(grad_input [B, D], grad_weight [D, V] view)`` times
    ``grad_output`` from the workspace of ``linear_cross_entropy_stats_keep``
    (the dW GEMM, then the dH GEMM)."""
    import ctypes

    from greyhound_b200 import _lib

    B, D = inputs.shape
    V = weight.shape[1]
    x = inputs.contiguous()
    w = _weight_vd(weight)
    dev = inputs.device
    lib = _lib.load()
    _lib.raise_pending(dev, "linear_cross_entropy backward")
    code = _lib.dtype_code(inputs.dtype)
    chunk = chunk_size_for(B, D, V, inputs.element_size())
    g = grad_output.reshape(1).float().contiguous() if grad_output is not None else None
    stream = _lib.stream_of(x)
    gw = torch.empty((V, D), dtype=weight.dtype, device=dev)
    band = (ctypes.c_void_p * 1)(gw.data_ptr())  # one band: this GPU's own gradient
    st = lib.gh_lce_dw_peers(x.data_ptr(), B, D, V, code, chunk, int(fp32_accum), _lib.ptr(g), band, 1,
                             -(-V // 256) * 256, 0, ws.data_ptr(), ws.numel(), stream)
    _lib.check(st, "linear_cross_entropy dW")
    gi = torch.empty((B, D), dtype=inputs.dtype, device=dev)
    st = lib.gh_lce_dh_last_chunk(w.data_ptr(), B, D, V, code, chunk, int(fp32_accum), 0, -1, _lib.ptr(g),
                                  gi.data_ptr(), ws.data_ptr(), ws.numel(), 0, stream)
    _lib.check(st, "linear_cross_entropy dH")
    _lib.raise_on_status(ws, "linear_cross_entropy backward")
    return gi, gw.T


def linear_cross_entropy_loss(
    inputs: Tensor,
    weight: Tensor,
    target: Tensor,
    z_loss_multiplier: float,
    ignore_index: int,
) -> tuple[Tensor, Tensor, Tensor]:
    """Forward only: ``(ce_sum, z_sum, n_valid)``, no gradient buffers."""
    _check(inputs, weight, target)
    if _tc_ok(inputs, weight):
        ce, z, n, _, _ = _tc_lce(inputs, weight, target, z_loss_multiplier, True, ignore_index,
                                 False, None, False)
        return ce, z, n
    from greyhound_b200.kernels.gemm import gemm_nt_fp32

    B, D = inputs.shape
    V = weight.shape[1]
    chunk = chunk_size_for(B, D, V, inputs.element_size())
    dev = inputs.device
    target = target.contiguous()
    ce_sum = torch.zeros((), dtype=torch.float32, device=dev)
    z_sum = torch.zeros((), dtype=torch.float32, device=dev)
    n_valid = torch.zeros((), dtype=torch.float32, device=dev)
    for s in range(0, B, chunk):
        e = min(s + chunk, B)
        logits = gemm_nt_fp32(inputs[s:e], weight.T).to(inputs.dtype)
        c, z, n = cross_entropy_with_grad(logits, target[s:e], z_loss_multiplier, ignore_index, None)
        ce_sum += c
        z_sum += z
        n_valid += n
    return ce_sum, z_sum, n_valid


def vocab_shard_stats(
    inputs: Tensor, weight_shard: Tensor, target: Tensor, vocab_start: int
) -> tuple[Tensor, object]:
    """Per-row statistics of one vocab shard: ``[rows, 3]`` fp32 ``(lse_shard, 1, x_t)``.

    ``(lse_shard, 1)`` is an exact (max, sum) pair since ``1 * exp(lse) =
    sum exp(logits)`` over the shard; ``x_t`` is the target logit, ``-inf`` when
    the row's target is not in this shard. Returns the statistics and an
    opaque state (the shard's logits) for ``vocab_shard_grads``.
    """
    from greyhound_b200 import _lib

    rows, D = inputs.shape
    Vs = weight_shard.shape[0]
    dev = inputs.device
    target = target.contiguous()
    if _tc_ok(inputs, weight_shard.T):
        x = inputs.contiguous()
        w = weight_shard.contiguous()
        lib = _lib.load()
        _lib.raise_pending(dev, "vocab_shard_stats")
        code = _lib.dtype_code(inputs.dtype)
        ws = _lib.workspace(lib.gh_lce_shard_workspace_bytes(rows, D, Vs, code), dev)
        stats = torch.empty((rows, 3), dtype=torch.float32, device=dev)
        st = lib.gh_lce_shard_stats(x.data_ptr(), w.data_ptr(), target.data_ptr(), rows, D, Vs, int(vocab_start),
                                    code, stats.data_ptr(), ws.data_ptr(), ws.numel(), _lib.stream_of(x))
        _lib.check(st, "vocab_shard_stats")
        return stats, ("tc", ws, x, w)
    # fp32 operands: emulated fp32 GEMM + the CE row kernel for the shard logsumexp
    from greyhound_b200.kernels.cross_entropy import cross_entropy_with_grad as _ce
    from greyhound_b200.kernels.gemm import gemm_nt_fp32

    logits = gemm_nt_fp32(inputs, weight_shard).to(inputs.dtype)
    lse = torch.empty(rows, dtype=torch.float32, device=dev)
    never = torch.full_like(target, -(1 << 62))
    _ce(logits, never, 0.0, -(1 << 62), None, lse_out=lse)
    local = target - vocab_start
    inside = (local >= 0) & (local < Vs)
    xt = logits.gather(1, local.clamp(0, Vs - 1)[:, None])[:, 0].float()
    xt = torch.where(inside, xt, torch.full_like(xt, float("-inf")))
    return torch.stack([lse, torch.ones_like(lse), xt], dim=1), ("torch", logits)


def vocab_shard_grads(
    inputs: Tensor,
    weight_shard: Tensor,
    state: object,
    target: Tensor,
    vocab_start: int,
    lse: Tensor,
    z_loss_multiplier: float,
    ignore_index: int,
    scale: Tensor,
    grad_input_hook=None,
) -> tuple[Tensor, Tensor]:
    """Gradient pass of one vocab shard given the global per-row logsumexp.

    Returns this shard's partial ``grad_input [rows, D]`` and ``grad_weight
    [V_shard, D]``. ``grad_input_hook(grad_input)`` (the cross-shard sum,
    returning an async work handle or None) is called as soon as the partial
    grad_input exists; the dW GEMM runs while it is in flight and the handle
    is waited on before returning.
    """
    from greyhound_b200 import _lib

    rows, D = inputs.shape
    Vs = weight_shard.shape[0]
    dev = inputs.device
    target = target.contiguous()
    lse = lse.contiguous().float()
    sc = scale.reshape(1).float().contiguous()
    lib = _lib.load()
    _lib.raise_pending(dev, "vocab_shard_grads")
    if state[0] == "tc":
        _, ws, x, w = state
        gi = torch.empty((rows, D), dtype=inputs.dtype, device=dev)
        gw = torch.empty((Vs, D), dtype=weight_shard.dtype, device=dev)
        stream = _lib.stream_of(x)
        # dlogits + partial dH first, so the dH all-reduce can overlap the dW GEMM
        st = lib.gh_lce_shard_grads(x.data_ptr(), w.data_ptr(), target.data_ptr(), lse.data_ptr(), rows, D, Vs,
                                    int(vocab_start), _lib.dtype_code(inputs.dtype), float(z_loss_multiplier),
                                    int(ignore_index), sc.data_ptr(), gi.data_ptr(), None, ws.data_ptr(),
                                    ws.numel(), stream)
        _lib.check(st, "vocab_shard_grads")
        work = grad_input_hook(gi) if grad_input_hook is not None else None
        sms = torch.cuda.get_device_properties(dev).multi_processor_count
        reserve = int(os.environ.get("GREYHOUND_B200_COMM_SMS", str(_COMM_SMS)))
        st = lib.gh_lce_shard_dw(x.data_ptr(), rows, D, Vs, _lib.dtype_code(inputs.dtype), gw.data_ptr(),
                                 ws.data_ptr(), ws.numel(), max(2, sms - reserve) if work is not None else 0,
                                 stream)
        _lib.check(st, "vocab_shard_grads dW")
        if work is not None:
            work.wait()
        return gi, gw
    logits = state[1]
    labels = torch.where(target == ignore_index, torch.full_like(target, -(1 << 62)), target)
    st = lib.gh_logits_grad(
        logits.data_ptr(), logits.data_ptr(), labels.data_ptr(), lse.data_ptr(), rows, Vs,
        _lib.dtype_code(logits.dtype), float(z_loss_multiplier), -(1 << 62), int(vocab_start),
        sc.data_ptr(), _lib.stream_of(logits),
    )
    _lib.check(st, "gh_logits_grad")
    from greyhound_b200.kernels.gemm import gemm_nt_fp32

    gi = gemm_nt_fp32(logits, weight_shard.T).to(inputs.dtype)
    work = grad_input_hook(gi) if grad_input_hook is not None else None
    gw = gemm_nt_fp32(logits.T, inputs.T).to(inputs.dtype)
    if work is not None:
        work.wait()
    return gi, gw
