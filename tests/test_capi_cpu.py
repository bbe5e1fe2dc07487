"""C-ABI library: it loads without a GPU and exports every symbol that
include/greyhound_b200.h declares; host-side validation raises the reference's
exception types. No compute calls (no GPU here)."""

import ctypes
import re
from pathlib import Path

import pytest
import torch

from greyhound_b200 import _lib

ROOT = Path(__file__).resolve().parent.parent


def declared_symbols() -> list[str]:
    names = []
    for h in sorted((ROOT / "include").glob("*.h")):
        names += re.findall(r"^GH_API\s+[\w\s\*]+?\b(gh_\w+)\s*\(", h.read_text(), flags=re.M)
    return names


def test_header_declares_entry_points():
    names = declared_symbols()
    for required in ("gh_ce_fwd_grad", "gh_sls_fwd", "gh_sls_bwd", "gh_last_error_string"):
        assert required in names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"


def test_python_signatures_cover_header():
    assert set(declared_symbols()) <= set(_lib.SIGNATURES), set(declared_symbols()) - set(_lib.SIGNATURES)


def test_no_device_calls_needed_for_metadata():
    lib = _lib.load()
    assert lib.gh_abi_version() >= 1
    assert lib.gh_workspace_status_offset() == 0
    assert lib.gh_launch_count() >= 0


def test_invalid_args_map_to_reference_exceptions():
    lib = _lib.load()
    # bad dtype code -> TypeError (reference: unsupported logits dtype)
    st = lib.gh_ce_fwd_grad(None, None, None, 4, 8, 99, 0.0, -100, 0, None, 1, 1, 1, None, 1, 1 << 20, None)
    with pytest.raises(TypeError):
        _lib.check(st, "x")
    # empty vocab -> ValueError
    st = lib.gh_sls_fwd(None, None, _lib.GH_I64, 4, 0, _lib.GH_BF16, None, _lib.GH_BF16, None, 1, 1 << 20, None)
    with pytest.raises(ValueError):
        _lib.check(st, "x")
    # too-small workspace -> RuntimeError
    need = lib.gh_ce_workspace_bytes(64, 1000, _lib.GH_BF16)
    st = lib.gh_ce_fwd_grad(8, 8, 8, 64, 1000, _lib.GH_BF16, 0.0, -100, 0, None, 8, 8, 8, None, 8, need - 1, None)
    with pytest.raises(RuntimeError):
        _lib.check(st, "x")


def test_python_validation_matches_reference_messages():
    from greyhound_b200.kernels.cross_entropy import cross_entropy_with_grad_kernel
    from greyhound_b200.kernels.logprobs import selective_log_softmax_kernel

    x = torch.zeros(4, 8)
    with pytest.raises(ValueError, match="expected 2D logits"):
        cross_entropy_with_grad_kernel(torch.zeros(8), torch.zeros(8, dtype=torch.long), 0.0, -100)
    with pytest.raises(ValueError, match="expected labels shape"):
        cross_entropy_with_grad_kernel(x, torch.zeros(3, dtype=torch.long), 0.0, -100)
    with pytest.raises(ValueError, match="same CUDA device"):
        cross_entropy_with_grad_kernel(x, torch.zeros(4, dtype=torch.long), 0.0, -100)
    with pytest.raises(ValueError, match="at least 2 dimensions"):
        selective_log_softmax_kernel(torch.zeros(8), torch.zeros((), dtype=torch.long))
    with pytest.raises(ValueError, match="same CUDA device"):
        selective_log_softmax_kernel(x, torch.zeros(4, dtype=torch.long))


def test_workspace_sizes_are_modest():
    lib = _lib.load()
    # the row kernels need O(rows) scratch, never O(rows * V)
    assert lib.gh_ce_workspace_bytes(65536, 151936, _lib.GH_BF16) < 4 << 20
    assert lib.gh_ce_workspace_bytes(16, 128256, _lib.GH_BF16) < 1 << 20
