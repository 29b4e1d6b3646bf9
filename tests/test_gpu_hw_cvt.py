"""The hardware E2M1 / E4M3 converters used by the BF16 fast path round exactly like the
library's software rounding (itself pinned to the reference by the golden tests), checked
exhaustively over every float32 in the ranges that reach them."""

import subprocess
import tempfile
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]


def test_hardware_fp4_fp8_converters_match_software_rounding():
    with tempfile.TemporaryDirectory() as tmp:
        exe = Path(tmp) / "hw_cvt_check"
        subprocess.run(["nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-O2", "-std=c++17",
                        f"-I{ROOT / 'qatfactory_b200' / 'csrc'}", str(ROOT / "tests" / "cuda" / "hw_cvt_check.cu"),
                        "-o", str(exe)], check=True)
        out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stdout + out.stderr
    assert "e2m1 mismatches 0" in out.stdout and "e4m3 mismatches 0" in out.stdout
