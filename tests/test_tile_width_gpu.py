"""Both GEMM tile widths stay parity-tested.

The library picks 256- or 512-column pair tiles per GEMM (512 for plain
16-bit stores, 256 for the linear-CE logits GEMM and fp32 epilogues), so a
default run exercises only one width per GEMM. GREYHOUND_B200_GEMM_WIDE is
read once per process; each width therefore reruns the GEMM and linear-CE
parity tests in a child process with the width forced.
"""

import os
import subprocess
import sys
from pathlib import Path

import pytest

from greyhound_b200.testing import requires_gpu

ROOT = Path(__file__).resolve().parent.parent


@requires_gpu
@pytest.mark.skipif("GREYHOUND_B200_GEMM_WIDE" in os.environ, reason="already inside a forced-width run")
@pytest.mark.parametrize("mode", ["0", "2"])
def test_parity_with_forced_tile_width(mode):
    env = dict(os.environ, GREYHOUND_B200_GEMM_WIDE=mode)
    res = subprocess.run(
        [sys.executable, "-m", "pytest", "-x", "-q", "-m", "gpu", "-p", "no:cacheprovider",
         "tests/test_gemm_gpu.py", "tests/test_chunked_linear_gpu.py"],
        cwd=ROOT, env=env, capture_output=True, text=True, timeout=900,
    )
    assert res.returncode == 0, res.stdout[-4000:] + res.stderr[-2000:]
