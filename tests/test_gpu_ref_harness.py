"""GPU: the reference's own CLI (src/sepia.c, built in place and linked
against libsepia_cuda.so instead of its Metal shim -- oracle/_ref/sepia_cuda)
runs its own GPU gates against this backend:
  --gpu-selftest      buffers / wrap_mmap / touch (src/sepia.c:4469-4548)
  --gpu-quants FIX..  bitwise dequant + matvec <= 2e-4 vs its qlinear
                      (src/sepia.c:5944-6061)
  --gpu-compare-attn  7 attention edge cases vs its attn_forward_chunk
                      (src/sepia.c:5217-5326)
"""
import subprocess
from pathlib import Path

import pytest

from golden_io import golden_files

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent
BIN = ROOT / "oracle" / "_ref" / "sepia_cuda"


@pytest.fixture(scope="module")
def sepia_bin(lib):
    if not BIN.exists():
        pytest.skip("oracle/_ref/sepia_cuda not built (needs the reference checkout at build time)")
    return str(BIN)


def run(args, timeout=300):
    r = subprocess.run(args, capture_output=True, text=True, timeout=timeout, cwd=str(ROOT))
    return r.returncode, r.stdout + r.stderr


def test_reference_gpu_selftest(sepia_bin):
    code, out = run([sepia_bin, "--metal", "--gpu-selftest"])
    assert code == 0 and "gpu selftest ok" in out, out


def test_reference_gpu_quants(sepia_bin):
    files = [str(p) for p in golden_files("sqfx")]
    code, out = run([sepia_bin, "--metal", "--gpu-quants", *files])
    assert code == 0 and "gpu-quants ok" in out, out
    assert out.count("dequant ok") >= 7, out


def test_reference_gpu_compare_attn(sepia_bin):
    code, out = run([sepia_bin, "--metal", "--gpu-compare-attn"], timeout=600)
    assert code == 0, out
    assert "FAIL" not in out, out
