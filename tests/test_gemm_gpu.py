"""tcgen05 GEMM (gh_gemm) against a torch fp32 matmul of the same bf16/fp16 values,
for all four operand-majorness combinations, odd shapes and both epilogue
addend/scale forms."""

import pytest
import torch

from greyhound_b200.kernels.gemm import gemm_nt
from greyhound_b200.testing import requires_gpu


def _view(x: torch.Tensor, mn_major: bool) -> torch.Tensor:
    # [R, K] view that is either row-major or the transpose of a row-major [K, R]
    return x.T.contiguous().T if mn_major else x.contiguous()


def _rel(a, b):
    return ((a.double() - b.double()).norm() / b.double().norm().clamp(min=1e-30)).item()


@requires_gpu
@pytest.mark.parametrize("a_mn", [False, True])
@pytest.mark.parametrize("b_mn", [False, True])
@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 512, 128), (200, 296, 136), (1000, 1304, 1000), (2048, 4096, 4096)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_gemm_matches_torch(a_mn, b_mn, M, N, K, dtype):
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N * 3 + K)
    a = torch.randn(M, K, device="cuda", generator=g).to(dtype)
    b = torch.randn(N, K, device="cuda", generator=g).to(dtype)
    ref = a.float() @ b.float().T
    out32 = gemm_nt(_view(a, a_mn), _view(b, b_mn), out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert _rel(out32, ref) < 1e-5 * K ** 0.5 + 1e-6
    out16 = gemm_nt(_view(a, a_mn), _view(b, b_mn))
    assert out16.dtype == dtype
    assert _rel(out16.float(), ref) < 1e-2


@requires_gpu
def test_gemm_addend_and_scale():
    g = torch.Generator(device="cuda").manual_seed(5)
    a = torch.randn(384, 512, device="cuda", generator=g).to(torch.bfloat16)
    b = torch.randn(640, 512, device="cuda", generator=g).to(torch.bfloat16)
    acc = torch.randn(384, 640, device="cuda", generator=g)
    scale = torch.tensor([0.25], device="cuda")
    ref = acc + 0.25 * (a.float() @ b.float().T)
    out = gemm_nt(a, b, out=acc, addend=acc, scale=scale)  # in-place accumulate
    assert out.data_ptr() == acc.data_ptr()
    assert _rel(out, ref) < 1e-5
    accb = torch.randn(384, 640, device="cuda", generator=g).to(torch.bfloat16)
    ref = accb.float() + a.float() @ b.float().T
    out = gemm_nt(a, b, out=accb, addend=accb)
    assert _rel(out.float(), ref) < 1e-2


@requires_gpu
def test_gemm_pipeline_timeout_returns_with_status():
    """Failure detection without a GPU fault: a GEMM whose loads never arrive
    gives up after a short bounded wait, reports GH_DEV_PIPELINE_TIMEOUT and
    returns; the context keeps working (a normal GEMM afterwards is correct)."""
    import time

    from greyhound_b200 import _lib

    lib = _lib.load()
    scratch = torch.zeros(128 * 1024, dtype=torch.uint8, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    t0 = time.time()
    st = lib.gh_gemm_selftest_stall(scratch.data_ptr(), scratch.numel(), status.data_ptr(), 50,
                                    torch.cuda.current_stream().cuda_stream)
    _lib.check(st, "selftest")
    torch.cuda.synchronize()
    assert time.time() - t0 < 30
    assert int(status.item()) & _lib.GH_DEV_PIPELINE_TIMEOUT
    a = torch.randn(256, 512, device="cuda").bfloat16()
    b = torch.randn(384, 512, device="cuda").bfloat16()
    out = gemm_nt(a, b, out_dtype=torch.float32)
    assert _rel(out, a.float() @ b.float().T) < 1e-5


@requires_gpu
@pytest.mark.parametrize("M,N,K", [(256, 384, 512), (300, 1000, 123), (1024, 512, 4096)])
def test_fp32_gemm_emulation_matches_fp64(M, N, K):
    """fp32 GEMMs of the fp32 linear-CE path run on the bf16 tcgen05 GEMM as
    six split-precision products, compared with fp64."""
    from greyhound_b200.kernels.gemm import gemm_nt_fp32

    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    a = torch.randn(M, K, device="cuda", generator=g)
    b = torch.randn(N, K, device="cuda", generator=g)
    ref = (a.double() @ b.double().T)
    got = gemm_nt_fp32(a, b)
    torch.backends.cuda.matmul.allow_tf32 = False
    f32 = a @ b.T
    err = (got.double() - ref).abs().max().item()
    err32 = (f32.double() - ref).abs().max().item()
    # measured: 0.6-4.5e-5 of max|C| (the tensor cores' fp32 accumulation
    # dominates), against 0.3-3e-6 for cuBLAS SGEMM and ~1e-3 for TF32
    assert err <= 1e-4 * ref.abs().max().item(), (err, err32)
    # transposed operand views and accumulation into an fp32 buffer
    acc = torch.randn(M, N, device="cuda", generator=g)
    ref2 = acc.double() + a.double() @ b.double().T
    got2 = gemm_nt_fp32(a.T.contiguous().T, b.T.contiguous().T, out=acc, addend=acc)
    assert (got2.double() - ref2).abs().max().item() <= 1e-4 * ref2.abs().max().item()
