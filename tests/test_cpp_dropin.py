"""Drop-in check: a host program written like the reference's benches compiles
against include/ (netcfg::, ll::TickBuffer, ll::dense_warp_rm_kernel<...>,
ll::launch_dense_mbyv_packed<...>, ll::dense_mbyv_kernel<...>, ll::PaddedCols, ll::Engine)
and, on a GPU, reproduces the reference's own golden output on every path."""
import os
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = os.path.join(ROOT, "tests", "cpp", "reference_style_host.cu")
LIBDIR = os.path.join(ROOT, "low_latency_inference_gpu_b200", "_lib")


def build(tmp_path):
    exe = str(tmp_path / "reference_style_host")
    cmd = ["nvcc", "-O2", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a", "-I", os.path.join(ROOT, "include"),
           SRC, "-o", exe, "-L", LIBDIR, "-lll_b200", "-Xlinker", f"-rpath,{LIBDIR}"]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    return exe


def test_reference_style_host_compiles(tmp_path):
    assert os.path.exists(build(tmp_path))


@pytest.mark.gpu
@pytest.mark.timeout(300)
def test_reference_style_host_runs_and_matches_golden(tmp_path, golden):
    exe = build(tmp_path)
    out = tmp_path / "out.bin"
    r = subprocess.run([exe, str(out)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    v = np.fromfile(out, np.float32)
    y_engine, y_warp, y_packed, y_mbyv = v[0], v[1], v[2], v[3]
    y3 = np.array(golden["ref_bench"]["y3"], np.uint32).view(np.float32)[0]
    for y in (y_engine, y_warp, y_packed, y_mbyv):
        assert abs(float(y) - float(y3)) <= 1e-5 * max(1.0, abs(float(y3)))
