"""Multi-GPU layer: data-parallel row sharding and vocab-parallel sharding of the
chunked linear cross-entropy (one process per GPU, ``torch.distributed``; NCCL
on GPUs, Gloo for CPU tests of the sharding arithmetic).

The reference is single-device only (src/greyhound/utils.py:4-7); these modes
are new. Both keep the reference's loss semantics: the loss is the sum over
all valid tokens of all ranks, divided by the *global* valid-token count for
``reduction="mean"``.

* Row sharding (``RowShardedLinearCrossEntropy``): each rank holds its own rows
  of ``inputs``/``target`` and a replica of ``weight``. One scalar all-reduce
  gives the global valid count before any gradient is written, so the
  ``1 / n_global`` scale is folded into the logits gradient. The weight
  gradient is summed across ranks by a reduce-scatter fused into the dW
  GEMM (tiles stored into the owning rank's buffer through CUDA IPC), a
  fixed-order sum on each owner and copy-engine copies of the reduced bands
  (``_row_sharded_band_exchange``); an NCCL all-reduce is the fallback for
  shapes that path does not take (several chunks, fp32, more than 8 ranks).
* Vocab sharding (``VocabShardedLinearCrossEntropy``): each rank holds rows
  ``[r*V/P, (r+1)*V/P)`` of ``weight`` and all rows of ``inputs``. Per row the
  ranks exchange (max, sum-exp, target-logit) with one all-gather, combine them
  into the exact global logsumexp, then each writes its slice of the logits
  gradient, its weight-gradient shard (no communication) and a partial input
  gradient that is summed with one all-reduce.
"""

from __future__ import annotations

from typing import Literal

import torch
import torch.distributed as dist
from torch import Tensor

from greyhound_b200.ops.scale import scale_by
from greyhound_b200.kernels import linear_cross_entropy as lce

__all__ = [
    "row_sharded_linear_cross_entropy",
    "vocab_sharded_linear_cross_entropy",
    "combine_vocab_stats",
    "shard_range",
]


def shard_range(total: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous near-equal split of ``[0, total)``; the first ``total % world`` shards get one extra."""
    base, rem = divmod(total, world)
    start = rank * base + min(rank, rem)
    return start, start + base + (1 if rank < rem else 0)


def _global_scale(target: Tensor, ignore_index: int, reduction: str, group) -> tuple[Tensor, Tensor]:
    n = (target != ignore_index).sum().to(torch.float32).reshape(1)
    if dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(n, group=group)
    if reduction == "mean":
        scale = 1.0 / n.clamp(min=1.0)
    elif reduction == "sum":
        scale = torch.ones_like(n)
    else:
        raise ValueError(f"Unsupported reduction: {reduction}")
    return n.reshape(()), scale


def _band_rows(V: int, world: int) -> int:
    """Rows per weight-gradient band: ceil(V / world) rounded up to the GEMM
    tile height (256)."""
    per_rank = -(-V // world)
    return -(-per_rank // 256) * 256


class _BandExchange:
    """Receive buffers of the weight-gradient reduce-scatter that the dW GEMM
    performs in its epilogue, shared between the ranks of one node with CUDA
    IPC (allocated once per group / device / shape and kept).

    The ``[V, D]`` gradient is cut into ``world`` row bands of ``band_rows``
    rows (a multiple of the GEMM tile height). Rank ``b`` owns band ``b``:
    ``recv[s]`` receives rank ``s``'s partial of that band (written by rank
    ``s``'s GEMM epilogue through the IPC mapping), and ``shard`` holds the
    reduced band, which the other ranks copy (copy engines, over NVLink)."""

    _cache: dict = {}

    @classmethod
    def get(cls, group, device, V, D, dtype):
        key = (id(group), device.index, V, D, dtype)
        ex = cls._cache.get(key)
        if ex is None:
            ex = cls(group, device, V, D, dtype)
            cls._cache[key] = ex
        return ex

    def __init__(self, group, device, V, D, dtype):
        import ctypes

        from greyhound_b200 import _lib

        self.lib = _lib.load()
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.group = group
        self.V, self.D, self.dtype = V, D, dtype
        self.band_rows = _band_rows(V, self.world)
        # one allocation (one IPC handle): world receive slots, then the reduced band
        self.buf = torch.empty((self.world + 1, self.band_rows, D), dtype=dtype, device=device)
        self.recv = self.buf[: self.world]
        self.shard = self.buf[self.world]
        h = ctypes.create_string_buffer(64)
        off = ctypes.c_size_t(0)
        _lib.check(self.lib.gh_ipc_get_handle(self.buf.data_ptr(), h, ctypes.byref(off)), "gh_ipc_get_handle")
        allh = [None] * self.world
        dist.all_gather_object(allh, (h.raw, off.value), group=group)
        slot = self.band_rows * D * self.buf.element_size()
        self.opened = []
        self.band_out = (ctypes.c_void_p * self.world)()
        self.shard_src = [0] * self.world
        for r, (hr, orr) in enumerate(allh):
            if r == self.rank:
                base = self.buf.data_ptr()
            else:
                pr = ctypes.c_void_p()
                _lib.check(self.lib.gh_ipc_open(hr, orr, ctypes.byref(pr)), "gh_ipc_open")
                self.opened.append((pr.value, orr))
                base = pr.value
            self.band_out[r] = base + self.rank * slot  # this rank's slot in rank r's receive buffer
            self.shard_src[r] = base + self.world * slot  # rank r's reduced band
        self.flag = torch.zeros(1, dtype=torch.float32, device=device)
        self.copy_stream = torch.cuda.Stream(device=device)

    def rows_of(self, b: int) -> int:
        return min(self.band_rows, self.V - b * self.band_rows)

    def barrier(self):
        """Stream-ordered barrier: returns on the host at once; the kernels
        queued after it run once every rank's earlier kernels have finished."""
        dist.all_reduce(self.flag, group=self.group)


def _dp_band_exchange_ok(inputs, weight_dv, world) -> bool:
    import os

    if os.environ.get("GREYHOUND_B200_DP_PEER", "1") in ("0", ""):
        return False
    if not (1 < world <= 8) or not lce._tc_ok(inputs, weight_dv):
        return False
    B, D = inputs.shape
    V = weight_dv.shape[1]
    return (B > 0 and (world - 1) * _band_rows(V, world) < V
            and lce.chunk_size_for(B, D, V, inputs.element_size()) >= B)


_DP_TIMING = __import__("os").environ.get("GREYHOUND_B200_DP_TIMING", "0") not in ("", "0")
DP_PHASES: list = []  # per backward: [(phase, CUDA event)], when _DP_TIMING


def dp_phase_summary() -> dict:
    """Mean ms of each band-exchange phase over the recorded backwards;
    synchronises. Each phase is measured from the mark it follows in stream
    order (the dH GEMM from the end of dW when it overlaps the exchange)."""
    torch.cuda.synchronize()
    acc: dict = {}
    for overlap, marks in DP_PHASES:
        d = dict(marks)
        ref = {"dw_gemm": "start", "barrier1": "dw_gemm", "sum_slots": "barrier1", "barrier2": "sum_slots",
               "copies_done": "barrier2", "dh_gemm": "dw_gemm" if overlap else "copies_done",
               "joined": "dh_gemm"}
        if not overlap:
            ref["dh_gemm"] = "barrier2"
        for name, ev in marks:
            if name in ref and ref[name] in d:
                acc.setdefault(name, []).append(d[ref[name]].elapsed_time(ev))
    DP_PHASES.clear()
    return {k: sum(v) / len(v) for k, v in acc.items()}


def _dp_overlap_sms() -> int:
    """SMs left to the weight-gradient exchange while the dH GEMM runs
    (GREYHOUND_B200_DP_OVERLAP_SMS, default 0: the exchange runs before dH).
    Measured at 2 GPUs with 8 SMs: the slot sum slows from 0.42 to 5.0 ms
    and dH by 0.5 ms, for the same step time (20.41 against 20.45 ms)."""
    import os

    return max(0, int(os.environ.get("GREYHOUND_B200_DP_OVERLAP_SMS", "0")))


def _exchange(ex, lib, gw, D, code, me, elt, cs, mark):
    """Barrier, fixed-order sum of this rank's band, barrier, and the copy-
    engine pulls of the other bands (on ``cs``); the stream-ordered part runs
    on the current stream."""
    from greyhound_b200 import _lib

    ex.barrier()  # every rank's slot of my band has arrived
    mark("barrier1", torch.cuda.current_stream())
    st = lib.gh_sum_slots(ex.recv.data_ptr(), ex.world, ex.band_rows * D, ex.rows_of(me), D, D, code,
                          ex.shard.data_ptr(), gw[me * ex.band_rows:].data_ptr(),
                          torch.cuda.current_stream().cuda_stream)
    _lib.check(st, "gh_sum_slots")
    mark("sum_slots", torch.cuda.current_stream())
    ex.barrier()  # every rank's reduced band is ready
    mark("barrier2", torch.cuda.current_stream())
    ready = torch.cuda.Event()
    ready.record()
    cs.wait_event(ready)
    for r in range(ex.world):
        if r != me:
            st = lib.gh_memcpy_async(gw[r * ex.band_rows:].data_ptr(), ex.shard_src[r], ex.rows_of(r) * D * elt,
                                     cs.cuda_stream)
            _lib.check(st, "gh_memcpy_async")
    mark("copies_done", cs)


def _band_exchange_grads(ws, inputs, weight_dv, grad_output, fp32_accum, group):
    """Backward of the data-parallel step (the forward kept the gradient
    operands in ``ws``, ``lce.linear_cross_entropy_stats_keep``). The weight
    gradient's all-reduce is a reduce-scatter fused into the dW GEMM's
    epilogue (each tile stored in the owner rank's receive slot), a
    fixed-order sum of the slots on each owner, and copies of the reduced
    bands between the ranks by the copy engines, overlapped with the
    input-gradient GEMM on all SMs. Both gradients come out multiplied by
    ``grad_output``."""
    from greyhound_b200 import _lib

    B, D = inputs.shape
    V = weight_dv.shape[1]
    dev = inputs.device
    ex = _BandExchange.get(group, dev, V, D, inputs.dtype)
    lib = ex.lib
    _lib.raise_pending(dev, "row_sharded_linear_cross_entropy backward")
    x = inputs.contiguous()
    w = lce._weight_vd(weight_dv)
    code = _lib.dtype_code(inputs.dtype)
    chunk = lce.chunk_size_for(B, D, V, inputs.element_size())
    gi = torch.empty((B, D), dtype=inputs.dtype, device=dev)
    gw = torch.empty((V, D), dtype=inputs.dtype, device=dev)
    g = grad_output.reshape(1).float().contiguous()
    stream = _lib.stream_of(x)
    marks = []

    def mark(name, st_=None):  # phase timing with CUDA events (GREYHOUND_B200_DP_TIMING=1)
        if _DP_TIMING:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record(st_)
            marks.append((name, ev))

    mark("start")
    # dW, each band's tiles stored straight into its owner's receive slot
    st = lib.gh_lce_dw_peers(x.data_ptr(), B, D, V, code, chunk, int(fp32_accum), g.data_ptr(), ex.band_out,
                             ex.world, ex.band_rows, (ex.rank + 1) % ex.world, ws.data_ptr(), ws.numel(), stream)
    _lib.check(st, "gh_lce_dw_peers")
    mark("dw_gemm")
    me = ex.rank
    cs = ex.copy_stream
    elt = gw.element_size()
    reserve = _dp_overlap_sms()
    if reserve > 0:
        # the exchange (barriers, slot sum, band copies) on its own stream
        # and `reserve` SMs, concurrent with the dH GEMM on the others
        ready = torch.cuda.Event()
        ready.record()
        cs.wait_event(ready)
        with torch.cuda.stream(cs):
            _exchange(ex, lib, gw, D, code, me, elt, cs, mark)
        sms = torch.cuda.get_device_properties(dev).multi_processor_count
        st = lib.gh_lce_dh_last_chunk(w.data_ptr(), B, D, V, code, chunk, int(fp32_accum), 0, -1, g.data_ptr(),
                                      gi.data_ptr(), ws.data_ptr(), ws.numel(), max(2, sms - reserve), stream)
    else:
        _exchange(ex, lib, gw, D, code, me, elt, cs, mark)
        # the input gradient on all SMs while the copy engines move the bands
        st = lib.gh_lce_dh_last_chunk(w.data_ptr(), B, D, V, code, chunk, int(fp32_accum), 0, -1, g.data_ptr(),
                                      gi.data_ptr(), ws.data_ptr(), ws.numel(), 0, stream)
    _lib.check(st, "linear_cross_entropy dH")
    mark("dh_gemm")
    torch.cuda.current_stream(dev).wait_stream(cs)
    mark("joined")
    gw.record_stream(cs)
    if _DP_TIMING:
        DP_PHASES.append((reserve > 0, marks))
    return gi, gw.T


class RowShardedLinearCrossEntropy(torch.autograd.Function):
    @staticmethod
    def forward(ctx, inputs, weight_dv, target, ignore_index, reduction, z_loss_multiplier, fp32_accum, group):
        n_global, scale = _global_scale(target, ignore_index, reduction, group)
        world = dist.get_world_size(group) if dist.is_initialized() else 1
        if _dp_band_exchange_ok(inputs, weight_dv, world):
            # loss now; both gradients and the weight-gradient exchange in the backward
            ce, zs, _, ws = lce.linear_cross_entropy_stats_keep(
                inputs, weight_dv, target, z_loss_multiplier, fp32_accum, ignore_index, False, grad_scale=scale)
            loss = (ce + z_loss_multiplier * zs).reshape(1)
            dist.all_reduce(loss, group=group)
            loss = (loss * scale).reshape(())
            ctx.band = (fp32_accum, group)
            ctx.save_for_backward(ws, inputs, weight_dv)
            return loss
        ctx.band = None
        hook = None
        if world > 1:
            def hook(grad_weight: Tensor):
                return dist.all_reduce(grad_weight, group=group, async_op=True)
        ce, zs, _, gi, gw = lce.linear_cross_entropy_with_grad(
            inputs, weight_dv, target, z_loss_multiplier, fp32_accum, ignore_index,
            grad_scale=scale, grad_weight_hook=hook,
        )
        loss = (ce + z_loss_multiplier * zs).reshape(1)
        if world > 1:
            dist.all_reduce(loss, group=group)
        loss = (loss * scale).reshape(())
        ctx.save_for_backward(gi, gw)
        return loss

    @staticmethod
    def backward(ctx, g):
        if ctx.band is not None:
            ws, inputs, weight_dv = ctx.saved_tensors
            gi, gw = _band_exchange_grads(ws, inputs, weight_dv, g, *ctx.band)
            return gi, gw, None, None, None, None, None, None
        gi, gw = ctx.saved_tensors
        return scale_by(gi, g), scale_by(gw, g), None, None, None, None, None, None


def row_sharded_linear_cross_entropy(
    inputs: Tensor,
    weight: Tensor,
    target: Tensor,
    ignore_index: int = -100,
    reduction: Literal["sum", "mean"] = "mean",
    z_loss_multiplier: float = 0.0,
    grad_weight_accum_dtype: Literal["fp32", "weight"] = "fp32",
    group=None,
) -> Tensor:
    """Data-parallel ``chunked_linear_cross_entropy``: this rank's rows, replicated ``weight [V, D]``.

    Returns the global loss (identical on every rank); ``weight.grad`` is the
    all-reduced global gradient, ``inputs.grad`` this rank's rows.
    """
    if grad_weight_accum_dtype not in ("fp32", "weight"):
        raise ValueError(f"grad_weight_accum_dtype must be either 'fp32' or 'weight', got {grad_weight_accum_dtype!r}")
    return RowShardedLinearCrossEntropy.apply(
        inputs, weight.T, target, ignore_index, reduction, z_loss_multiplier,
        grad_weight_accum_dtype == "fp32", group,
    )


def combine_vocab_stats(stats: Tensor) -> tuple[Tensor, Tensor]:
    """Combine per-shard row statistics into the global logsumexp and target logit.

    ``stats`` is ``[P, rows, 3]`` fp32 holding, for every vocab shard, the row
    max ``m``, ``s = sum exp(x - m)`` over the shard and the target logit (or
    ``-inf`` when the target is not in that shard). Exact, order-independent
    merge: ``lse = M + log(sum_p s_p exp(m_p - M))`` with ``M = max_p m_p``.
    """
    m, s, xt = stats[..., 0], stats[..., 1], stats[..., 2]
    M = m.max(dim=0).values
    Msafe = torch.where(torch.isfinite(M), M, torch.zeros_like(M))
    total = (s * torch.exp(m - Msafe)).sum(dim=0)
    lse = Msafe + torch.log(total)
    x_target = xt.max(dim=0).values
    return lse, x_target


class VocabShardedLinearCrossEntropy(torch.autograd.Function):
    @staticmethod
    def forward(ctx, inputs, weight_shard, target, vocab_start, ignore_index, reduction, z_loss_multiplier, group):
        world = dist.get_world_size(group) if dist.is_initialized() else 1
        valid = target != ignore_index
        n = valid.sum().to(torch.float32)
        if reduction == "mean":
            scale = 1.0 / n.clamp(min=1.0)
        elif reduction == "sum":
            scale = torch.ones_like(n)
        else:
            raise ValueError(f"Unsupported reduction: {reduction}")
        stats, state = lce.vocab_shard_stats(inputs, weight_shard, target, vocab_start)
        if world > 1:
            gathered = [torch.empty_like(stats) for _ in range(world)]
            dist.all_gather(gathered, stats, group=group)
            all_stats = torch.stack(gathered)
        else:
            all_stats = stats[None]
        lse, x_t = combine_vocab_stats(all_stats)
        ce = torch.where(valid, lse - x_t, torch.zeros_like(lse)).sum()
        zs = torch.where(valid, lse * lse, torch.zeros_like(lse)).sum()
        loss = (ce + z_loss_multiplier * zs) * scale
        hook = None
        if world > 1:
            def hook(gi_partial: Tensor):
                return dist.all_reduce(gi_partial, group=group, async_op=True)
        gi, gw = lce.vocab_shard_grads(
            inputs, weight_shard, state, target, vocab_start, lse, z_loss_multiplier, ignore_index, scale,
            grad_input_hook=hook,
        )
        ctx.save_for_backward(gi, gw)
        return loss

    @staticmethod
    def backward(ctx, g):
        gi, gw = ctx.saved_tensors
        return scale_by(gi, g), scale_by(gw, g), None, None, None, None, None, None


def vocab_sharded_linear_cross_entropy(
    inputs: Tensor,
    weight_shard: Tensor,
    target: Tensor,
    vocab_start: int,
    ignore_index: int = -100,
    reduction: Literal["sum", "mean"] = "mean",
    z_loss_multiplier: float = 0.0,
    group=None,
) -> Tensor:
    """Vocab-parallel ``chunked_linear_cross_entropy``.

    ``weight_shard`` is this rank's ``[V_local, D]`` rows of the ``[V, D]``
    weight, starting at vocab id ``vocab_start``; ``inputs``/``target`` are the
    full (replicated) rows. Returns the global loss on every rank;
    ``weight_shard.grad`` is this shard's gradient and ``inputs.grad`` the full
    (all-reduced) input gradient.
    """
    return VocabShardedLinearCrossEntropy.apply(
        inputs, weight_shard, target, int(vocab_start), ignore_index, reduction, z_loss_multiplier, group
    )
