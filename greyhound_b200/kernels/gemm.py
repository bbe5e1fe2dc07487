"""tcgen05 GEMM (sm_100a) through the C-ABI: ``out = scale * A @ B.T (+ addend)``.

``A`` is an ``[M, K]`` and ``B`` an ``[N, K]`` tensor view; each may be
row-major (K contiguous) or the transpose of a row-major matrix (M / N
contiguous). bf16 / fp16 operands, fp32 accumulation, output in fp32 or the
operand dtype. Used for the GEMMs of the generic chunked-loss path
(src/greyhound/ops/chunked_linear_loss.py:82,94,95-101).
"""

from __future__ import annotations

import torch
from torch import Tensor

from greyhound_b200 import _lib

__all__ = ["gemm_nt", "gemm_nt_fp32", "supports"]


def _operand(t: Tensor) -> tuple[Tensor, int, int]:
    """(tensor, leading dimension, mn_major) for an [R, K] view."""
    if t.stride(1) == 1 and t.stride(0) >= t.shape[1]:
        return t, t.stride(0), 0
    if t.stride(0) == 1 and t.stride(1) >= t.shape[0]:
        return t, t.stride(1), 1
    t = t.contiguous()
    return t, t.stride(0), 0


def supports(*tensors: Tensor) -> bool:
    """True when the tensors can go through the tcgen05 GEMM (dtype, device, alignment)."""
    for t in tensors:
        if not t.is_cuda or t.dtype not in (torch.bfloat16, torch.float16):
            return False
    return True


def gemm_nt(
    a: Tensor,
    b: Tensor,
    out_dtype: torch.dtype | None = None,
    out: Tensor | None = None,
    addend: Tensor | None = None,
    scale: Tensor | None = None,
) -> Tensor:
    if a.ndim != 2 or b.ndim != 2 or a.shape[1] != b.shape[1]:
        raise ValueError(f"gemm_nt expects A [M, K] and B [N, K], got {tuple(a.shape)} and {tuple(b.shape)}")
    if a.dtype != b.dtype or a.dtype not in (torch.bfloat16, torch.float16):
        raise TypeError(f"gemm_nt operands must both be bf16 or fp16, got {a.dtype} and {b.dtype}")
    M, K = a.shape
    N = b.shape[0]
    out_dtype = out_dtype or (out.dtype if out is not None else a.dtype)
    if out is None:
        out = torch.empty((M, N), dtype=out_dtype, device=a.device)
    if out.shape != (M, N) or out.stride(1) != 1:
        raise ValueError("out must be a row-major [M, N] tensor")
    a, lda, amn = _operand(a)
    b, ldb, bmn = _operand(b)
    # TMA wants 16-byte aligned bases and row pitches; re-lay out if needed.
    if (a.data_ptr() % 16) or (lda * a.element_size()) % 16:
        a, lda, amn = a.contiguous(), K, 0
        if (lda * a.element_size()) % 16:
            raise ValueError("K must be a multiple of 8 for the tcgen05 GEMM")
    if (b.data_ptr() % 16) or (ldb * b.element_size()) % 16:
        b, ldb, bmn = b.contiguous(), K, 0
    if addend is not None and (addend.shape != (M, N) or addend.stride(1) != 1 or addend.dtype != out.dtype):
        raise ValueError("addend must be a row-major [M, N] tensor of the output dtype")
    lib = _lib.load()
    st = lib.gh_gemm(
        a.data_ptr(), lda, amn, b.data_ptr(), ldb, bmn, M, N, K, _lib.dtype_code(a.dtype),
        out.data_ptr(), out.stride(0), _lib.dtype_code(out.dtype),
        _lib.ptr(addend), addend.stride(0) if addend is not None else 0,
        _lib.ptr(scale), None, _lib.stream_of(out),
    )
    _lib.check(st, "gemm_nt")
    return out


def _split3(t: Tensor, kp: int) -> tuple[Tensor, Tensor, Tensor]:
    """fp32 [R, K] -> three bf16 [R, kp] pieces t1 + t2 + t3 = t (to ~2^-24
    relative; zero padding from K to kp)."""
    t = t.float()
    t1 = t.bfloat16()
    r = t - t1.float()
    t2 = r.bfloat16()
    t3 = (r - t2.float()).bfloat16()
    if kp != t.shape[1]:
        pad = lambda u: torch.nn.functional.pad(u, (0, kp - t.shape[1]))  # noqa: E731
        t1, t2, t3 = pad(t1), pad(t2), pad(t3)
    return t1, t2, t3


def gemm_nt_fp32(a: Tensor, b: Tensor, out: Tensor | None = None, addend: Tensor | None = None) -> Tensor:
    """fp32 ``a @ b.T (+ addend)`` on the bf16 tcgen05 GEMM: each operand is
    split into three bf16 pieces (x = x1 + x2 + x3, 24 significand bits) and
    the six products whose magnitude reaches 2^-24 of the result (a1b1, a1b2,
    a2b1, a1b3, a2b2, a3b1) are summed in the GEMM's fp32 accumulator as one
    GEMM over a 6x longer K (the pieces concatenated along K): the usual
    split-precision emulation of single precision on lower-precision tensor
    cores. Measured error against fp64: 0.6-4.5e-5 of max|C| for K up to
    4096 (the tensor cores' accumulation dominates), where cuBLAS SGEMM gives
    0.3-3e-6 and a TF32 GEMM about 1e-3 (PyTorch's default fp32 matmul does
    not round to TF32). It replaces the cuBLAS SGEMMs of the fp32 operands."""
    if a.ndim != 2 or b.ndim != 2 or a.shape[1] != b.shape[1]:
        raise ValueError(f"gemm_nt_fp32 expects A [M, K] and B [N, K], got {tuple(a.shape)} and {tuple(b.shape)}")
    M, K = a.shape
    kp = -(-K // 8) * 8
    a1, a2, a3 = _split3(a, kp)
    b1, b2, b3 = _split3(b, kp)
    A = torch.cat([a1, a1, a2, a1, a2, a3], dim=1)
    B = torch.cat([b1, b2, b1, b3, b2, b1], dim=1)
    del a1, a2, a3, b1, b2, b3
    return gemm_nt(A, B, out_dtype=torch.float32, out=out, addend=addend)
