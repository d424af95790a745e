"""The C ABI from a C++ host (tests/cabi/consumer.cpp): compiled with the
host compiler against include/scao_b200.h and the built library, run as a
separate process, no Python or torch on its side."""
import os
import shutil
import subprocess

import pytest

from scao_b200 import _lib

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_cpp_consumer(tmp_path):
    cxx = shutil.which("g++") or shutil.which("c++")
    if cxx is None:
        pytest.skip("no C++ compiler")
    so = _lib.lib()._name
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    exe = tmp_path / "consumer"
    subprocess.check_call([cxx, "-O2", "-std=c++17", os.path.join(ROOT, "tests", "cabi", "consumer.cpp"),
                           "-I", os.path.join(ROOT, "include"), "-I", os.path.join(cuda, "include"),
                           so, "-L", os.path.join(cuda, "lib64"), "-lcudart",
                           f"-Wl,-rpath,{os.path.dirname(so)}", f"-Wl,-rpath,{os.path.join(cuda, 'lib64')}",
                           "-o", str(exe)])
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stderr
    assert "CABI OK" in out.stdout
