"""The streaming GEMV's 32-weight K-quant lane tasks (gemv_dev.cuh kq_*
helpers) decode every weight of a row exactly as ggml's dequantize_row_q5_K /
_q6_K do: tests/kquant_lanes_host.cu is built with nvcc (host code only) and
its per-task decode is compared bit for bit with the oracle.  No GPU."""
import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest

import vvq2_oracle as O

ROOT = Path(__file__).resolve().parent.parent
NVCC = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"


@pytest.fixture(scope="module")
def harness(tmp_path_factory):
    if not Path(NVCC).exists():
        pytest.skip("nvcc not available")
    out = tmp_path_factory.mktemp("kq") / "kq_host"
    r = subprocess.run([NVCC, "-std=c++17", "-O1", "-I", str(ROOT / "vibevoice.cpp_b200" / "csrc"),
                        str(ROOT / "tests" / "kquant_lanes_host.cu"), "-o", str(out)],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-2000:]
    return out


@pytest.mark.parametrize("qt", [O.Q5_K, O.Q6_K])
def test_lane_tasks_decode_like_ggml(harness, tmp_path, qt):
    rng = np.random.default_rng(100 + qt)
    cols = 2048
    w = (rng.standard_normal((1, cols)) * 0.05).astype(np.float32)
    raw = np.ascontiguousarray(O.quantize(qt, w)).reshape(-1)
    src, dst = tmp_path / "raw.bin", tmp_path / "out.bin"
    raw.tofile(src)
    r = subprocess.run([str(harness), str(qt), str(cols), str(src), str(dst)], capture_output=True)
    assert r.returncode == 0
    got = np.fromfile(dst, np.float32)
    ref = np.asarray(O.dequantize(qt, raw, cols), np.float32)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
