"""The C++ drop-in class `lite_ssm::MetalOps` (include/lite_ssm_b200/ops.hpp, built as
lite-ssm_b200/liblite_ssm_ops.so over the C ABI): a C++ test program is compiled against
the header and run. Without a GPU it checks that construction reports the missing device
as std::runtime_error; on a B200 it runs the kernel list of the reference's
tests/test_metal_ops.cpp:31-49, ops against host reference loops, batching and the
dims-check exceptions (tests/cpp/test_metal_ops_shim.cpp)."""

import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
PKG = ROOT / "lite-ssm_b200"


@pytest.fixture(scope="module")
def shim_exe(tmp_path_factory):
    sys.path.insert(0, str(PKG))
    import build as B   # noqa: E402

    if not B.LIB.exists():
        B.build()
    B.build_cpp_shim()
    exe = tmp_path_factory.mktemp("shim") / "test_metal_ops_shim"
    cmd = [os.environ.get("CXX", "g++"), "-O1", "-std=c++17", f"-I{ROOT / 'include'}",
           str(ROOT / "tests" / "cpp" / "test_metal_ops_shim.cpp"), "-o", str(exe), f"-L{PKG}", "-llite_ssm_ops",
           "-llssm_cuda", f"-Wl,-rpath,{PKG}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return exe


def test_shim_builds_and_reports_missing_device(shim_exe):
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present; the gpu test covers this binary")
    r = subprocess.run([str(shim_exe), "cpu"], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "PASS" in r.stdout


@pytest.mark.gpu
def test_shim_ops_on_gpu(shim_exe):
    r = subprocess.run([str(shim_exe), "gpu"], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "PASS" in r.stdout
