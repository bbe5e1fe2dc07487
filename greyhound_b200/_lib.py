"""ctypes binding of the C-ABI library ``_lib/libgreyhound_b200.so``.

Every compute entry point of greyhound_b200 goes through here. There is no
CPU fallback: if the library is missing or the tensors are not on a CUDA
device, calls raise. Error codes returned by the library are mapped to the
exception types the reference raises for the same conditions
(src/greyhound/kernels/cross_entropy.py:173-184: ValueError for shapes,
devices and layouts, TypeError for dtypes).
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libgreyhound_b200.so"

GH_F16, GH_BF16, GH_F32, GH_I32, GH_I64 = 0, 1, 2, 3, 4
GH_OK, GH_EINVAL, GH_ETYPE, GH_ECUDA, GH_EWORKSPACE, GH_EUNSUPPORTED = 0, 1, 2, 3, 4, 5
GH_DEV_BAD_LABEL = 1
GH_DEV_PIPELINE_TIMEOUT = 4

DTYPE_CODE = {
    torch.float16: GH_F16,
    torch.bfloat16: GH_BF16,
    torch.float32: GH_F32,
    torch.int32: GH_I32,
    torch.int64: GH_I64,
}

_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int
_f32 = ctypes.c_float
_sz = ctypes.c_size_t

# name -> (restype, argtypes); must match include/greyhound_b200.h
SIGNATURES: dict[str, tuple] = {
    "gh_abi_version": (_i32, []),
    "gh_last_error_string": (ctypes.c_char_p, []),
    "gh_launch_count": (ctypes.c_longlong, []),
    "gh_workspace_status_offset": (_sz, []),
    "gh_ce_workspace_bytes": (_sz, [_i64, _i64, _i32]),
    "gh_ce_fwd_grad": (
        _i32,
        [_vp, _vp, _vp, _i64, _i64, _i32, _f32, _i64, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _vp],
    ),
    "gh_ce_noalloc_scratch_bytes": (_sz, []),
    "gh_ce_fwd_grad_noalloc": (
        _i32,
        [_vp, _vp, _vp, _i64, _i64, _i32, _f32, _i64, _i32, _vp, _vp, _vp, _vp, _vp, _vp],
    ),
    "gh_sls_workspace_bytes": (_sz, [_i64, _i64, _i32]),
    "gh_sls_fwd": (_i32, [_vp, _vp, _i32, _i64, _i64, _i32, _vp, _i32, _vp, _vp, _sz, _vp]),
    "gh_sls_bwd": (_i32, [_vp, _vp, _i32, _vp, _vp, _i32, _i64, _i64, _i32, _vp, _vp]),
    "gh_logits_grad": (_i32, [_vp, _vp, _vp, _vp, _i64, _i64, _i32, _f32, _i64, _i64, _vp, _vp]),
    "gh_lce_workspace_bytes": (_sz, [_i64, _i64, _i64, _i64, _i32, _i32]),
    "gh_lce_loss_workspace_bytes": (_sz, [_i64, _i64, _i64, _i64, _i32]),
    "gh_lce_fwd_bwd": (
        _i32,
        [_vp, _vp, _vp, _i64, _i64, _i64, _i32, _f32, _i64, _i32, _vp, _i64, _i32, _i32,
         _vp, _vp, _vp, _vp, _vp, _vp, _sz, _vp],
    ),
    "gh_lce_dh_last_chunk": (
        _i32, [_vp, _i64, _i64, _i64, _i32, _i64, _i32, _i64, _i64, _vp, _vp, _vp, _sz, _i32, _vp]
    ),
    "gh_gemm": (
        _i32,
        [_vp, _i64, _i32, _vp, _i64, _i32, _i64, _i64, _i64, _i32, _vp, _i64, _i32, _vp, _i64, _vp, _vp, _vp],
    ),
    "gh_scale": (_i32, [_vp, _vp, _i64, _i32, _vp, _vp]),
    "gh_gemm_selftest_stall": (_i32, [_vp, _sz, _vp, _i32, _vp]),
    "gh_lce_shard_workspace_bytes": (_sz, [_i64, _i64, _i64, _i32]),
    "gh_lce_shard_stats": (_i32, [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _i32, _vp, _vp, _sz, _vp]),
    "gh_lce_shard_dw": (_i32, [_vp, _i64, _i64, _i64, _i32, _vp, _vp, _sz, _i32, _vp]),
    "gh_lce_shard_grads": (
        _i32,
        [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i32, _f32, _i64, _vp, _vp, _vp, _vp, _sz, _vp],
    ),
    "gh_lce_dw_peers": (
        _i32, [_vp, _i64, _i64, _i64, _i32, _i64, _i32, _vp, ctypes.POINTER(_vp), _i32, _i64, _i32, _vp, _sz, _vp]
    ),
    "gh_sum_slots": (_i32, [_vp, _i32, _i64, _i64, _i64, _i64, _i32, _vp, _vp, _vp]),
    "gh_ipc_get_handle": (_i32, [_vp, _vp, ctypes.POINTER(_sz)]),
    "gh_ipc_open": (_i32, [_vp, _sz, ctypes.POINTER(_vp)]),
    "gh_ipc_close": (_i32, [_vp, _sz]),
    "gh_memcpy_async": (_i32, [_vp, _vp, _sz, _vp]),
    "gh_take_device_errors": (_i32, [_i32]),
    "gh_ce_noalloc_status": (_i32, [ctypes.POINTER(ctypes.c_int), _vp]),
    "gh_profile_enable": (None, [_i32]),
    "gh_profile_read": (_i32, [ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_longlong), _i32, _i32]),
}
GH_LCE_DEFER_LAST_DH = 1
GH_LCE_KEEP_DW_OPERAND = 2
GH_LCE_GRADS_LATER = 4
PROF_CLASSES = ("gemm_logits_ce", "gemm_dw", "gemm_dh", "glue", "rows", "gemm_other")

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class GreyhoundLibraryError(RuntimeError):
    pass


def load() -> ctypes.CDLL:
    """Load (once) and return the C-ABI library. Raises if it was not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise GreyhoundLibraryError(
                    f"greyhound_b200 CUDA library not found at {LIB_PATH}; build it with "
                    "`python -m greyhound_b200.build` (there is no CPU fallback)"
                )
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def last_error() -> str:
    msg = load().gh_last_error_string()
    return msg.decode() if msg else ""


def check(status: int, what: str) -> None:
    if status == GH_OK:
        return
    msg = f"{what}: {last_error()}"
    if status == GH_EINVAL:
        raise ValueError(msg)
    if status == GH_ETYPE:
        raise TypeError(msg)
    raise GreyhoundLibraryError(msg)


def launch_count() -> int:
    return int(load().gh_launch_count())


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_of(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return DTYPE_CODE[dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype: {dtype}") from None


def workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)


def device_status(ws: torch.Tensor) -> int:
    """Read the device status word of a workspace (synchronises the stream)."""
    off = int(load().gh_workspace_status_offset())
    return int(ws[off : off + 4].view(torch.int32).item())


def profile_enable(on: bool) -> None:
    load().gh_profile_enable(1 if on else 0)


def profile_read(reset: bool = True) -> dict[str, tuple[float, int]]:
    """{class: (total_ms, launches)} of the event-timed launches (synchronises)."""
    n = len(PROF_CLASSES)
    ms = (ctypes.c_double * n)()
    cnt = (ctypes.c_longlong * n)()
    check(load().gh_profile_read(ms, cnt, n, 1 if reset else 0), "profile_read")
    return {PROF_CLASSES[i]: (ms[i], cnt[i]) for i in range(n)}


def scaled(t: torch.Tensor, g: torch.Tensor) -> torch.Tensor:
    """``t * g`` for a device scalar ``g`` (new tensor, same strides as ``t``)."""
    if not t.is_cuda:
        raise ValueError("expected a CUDA tensor (greyhound_b200 has no CPU path)")
    if t.numel() == 0 or t.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        return t * g
    if not (t.is_contiguous() or t.T.is_contiguous()) or t.data_ptr() % 16:
        return t * g
    raise_pending(t.device, "backward")
    out = torch.empty_like(t)  # preserves the (possibly transposed) dense layout
    gf = g.detach().reshape(1).to(torch.float32)
    check(load().gh_scale(t.data_ptr(), out.data_ptr(), t.numel(), dtype_code(t.dtype), gf.data_ptr(),
                          stream_of(t)), "scale")
    return out


CHECK_STATUS = os.environ.get("GREYHOUND_B200_CHECK", "0") not in ("", "0")


def take_device_errors(device: torch.device | int | None = None) -> int:
    """Read and clear the sticky device-error bits of a device (no sync).

    Every library call ends by OR-ing its workspace status word into a
    per-device slot of pinned host memory on the GPU; this returns the bits
    that calls which have already run on the GPU left there."""
    if device is None:
        idx = torch.cuda.current_device()
    elif isinstance(device, int):
        idx = device
    else:
        idx = device.index if device.index is not None else torch.cuda.current_device()
    return int(load().gh_take_device_errors(idx))


def _raise_bits(bits: int, what: str) -> None:
    if bits & GH_DEV_BAD_LABEL:
        raise ValueError(f"{what}: a target / index outside [0, vocab) that is not ignore_index "
                         "(recorded on the device by an earlier greyhound_b200 call)")
    if bits:
        raise GreyhoundLibraryError(f"{what}: device status {bits:#x} (a GEMM pipeline wait timed out "
                                    "in an earlier greyhound_b200 call; its results are not valid)")


def raise_pending(device: torch.device, what: str) -> None:
    """Raise for problems that earlier calls on ``device`` recorded on the GPU:
    ValueError for a label outside [0, V), RuntimeError for a pipeline timeout.
    Called on entry to every op and in the autograd backward; it does not
    synchronise, so a problem surfaces at the first call after the GPU has
    run the call that recorded it."""
    bits = take_device_errors(device)
    if bits:
        _raise_bits(bits, what)


def raise_on_status(ws: torch.Tensor, what: str) -> None:
    """With GREYHOUND_B200_CHECK=1: synchronise and raise at once if the
    kernels of the last call recorded a problem in the workspace status word
    (a label outside [0, V): ValueError; a pipeline timeout: RuntimeError).
    Without it the same bits surface through ``raise_pending`` on the next
    call, without a host sync."""
    if not CHECK_STATUS:
        return
    st = device_status(ws)
    take_device_errors(ws.device)  # reported here; do not report it twice
    _raise_bits(st, what)
