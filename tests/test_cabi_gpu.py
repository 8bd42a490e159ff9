"""The six reference custom-call targets called from C++ through the C ABI
with the reference's operand order and dtypes (f32 attention operands and
results, bf16 -> f32 GEMM, f32 CE): tests/cabi/reference_targets.cc is
compiled with g++ against include/nl_ops.h and libnl_ops.so and run; it checks
every result against a double-precision host computation."""
import shutil
import subprocess
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]


def test_reference_targets_from_cpp(cuda, tmp_path):
    from nlearn_b200 import _lib
    cxx = shutil.which("g++")
    if cxx is None:
        pytest.skip("g++ not available")
    cuda_home = Path("/usr/local/cuda")
    exe = tmp_path / "reference_targets"
    cmd = [cxx, "-O2", "-std=c++17", "-I", str(ROOT / "include"), "-I", str(cuda_home / "include"),
           str(ROOT / "tests" / "cabi" / "reference_targets.cc"), "-L", str(_lib.LIB_PATH.parent), "-l:libnl_ops.so",
           "-L", str(cuda_home / "lib64"), "-lcudart", f"-Wl,-rpath,{_lib.LIB_PATH.parent}", "-o", str(exe)]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.count("PASS") == 7
