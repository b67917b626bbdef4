"""The Q8_0 block scale, its reciprocal and the code rounding used by every
quantising kernel (kernrt_b200/csrc/q8_math.cuh) agree with CUDA's correctly
rounded division and with the float-clamp form of quant.rs:871 on every one of
the 2^32 f32 inputs, and the kernels' clamp-free codes stay within [-127, 127]
wherever they skip the clamp.  The check is compiled with the kernels' own flags and run
on the GPU."""
import os
import shutil
import subprocess

import pytest

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def test_q8_block_math_is_exact_on_every_f32(tmp_path):
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    exe = tmp_path / "q8_math_check"
    subprocess.run([nvcc, "-O3", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a", "-fmad=false",
                    "-o", str(exe), os.path.join(HERE, "cuda", "q8_math_check.cu")], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    for what in ("q8_scale", "q8_inv", "q8_code", "q8_inv_block", "q8_round bound"):
        assert f"{what} mismatches 0" in r.stdout, r.stdout
