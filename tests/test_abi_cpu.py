"""The C-ABI library loads without a GPU and exports every symbol that
include/scao_b200.h declares; the Python binding covers all of them."""
import ctypes
import os
import re

from scao_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared():
    src = open(os.path.join(ROOT, "include", "scao_b200.h")).read()
    return sorted(set(re.findall(r"SCAO_API\s+[\w\s\*]+?\b(scao_\w+)\s*\(", src)))


def test_header_declares_entry_points():
    names = declared()
    assert "scao_plan_step" in names and "scao_int8_ema_update_noalloc" in names
    assert len(names) >= 20


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(_lib.lib()._name)
    missing = [n for n in declared() if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_header():
    assert sorted(_lib.SIGNATURES) == declared()


def test_struct_layouts():
    _lib.check_layout()
    # ScaoPlanDev: 10 int32 header fields then pointers
    assert ctypes.sizeof(_lib.PlanDev) % 8 == 0


def test_host_only_queries():
    L = _lib.lib()
    assert L.scao_int8_ema_scratch_bytes(1000) >= 4000
    assert L.scao_fused_precond_scratch_bytes(64, 48, 8) > 0
    assert L.scao_int8_ema_update_noalloc_max_n() == 1 << 20
    assert b"sm_100a" in L.scao_version()


def test_struct_layouts_match_header(tmp_path):
    """Compile a probe against include/scao_b200.h with the host C compiler
    and compare every struct size and the PlanDev / FilterDev field offsets
    with the ctypes / numpy mirrors."""
    import shutil
    import subprocess
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        import pytest
        pytest.skip("no host C compiler")
    fields_plan = [f for f, _ in _lib.PlanDev._fields_]
    fields_filt = [f for f, _ in _lib.FilterDev._fields_]
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "scao_b200.h"',
             'int main(void) {']
    for t in ("ScaoParam", "ScaoParamStep", "ScaoLeaf", "ScaoChunk", "ScaoStrip", "ScaoFilterParam",
              "ScaoFilterDev", "ScaoPlanDev"):
        lines.append(f'printf("size {t} %zu\\n", sizeof({t}));')
    for f in fields_plan:
        lines.append(f'printf("plan {f} %zu\\n", offsetof(ScaoPlanDev, {f}));')
    for f in fields_filt:
        lines.append(f'printf("filt {f} %zu\\n", offsetof(ScaoFilterDev, {f}));')
    for f in _lib.FILTER_PARAM_DT.names:
        lines.append(f'printf("fparam {f} %zu\\n", offsetof(ScaoFilterParam, {f}));')
    lines.append("return 0; }")
    src = tmp_path / "probe.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "probe"
    subprocess.check_call([cc, "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)])
    out = subprocess.check_output([str(exe)]).decode().split("\n")
    got = {tuple(l.split()[:2]): int(l.split()[2]) for l in out if l.strip()}
    assert got[("size", "ScaoParam")] == _lib.PARAM_DT.itemsize
    assert got[("size", "ScaoParamStep")] == _lib.STEP_DT.itemsize
    assert got[("size", "ScaoLeaf")] == _lib.LEAF_DT.itemsize
    assert got[("size", "ScaoChunk")] == _lib.CHUNK_DT.itemsize
    assert got[("size", "ScaoStrip")] == _lib.STRIP_DT.itemsize
    assert got[("size", "ScaoFilterParam")] == _lib.FILTER_PARAM_DT.itemsize
    assert got[("size", "ScaoFilterDev")] == ctypes.sizeof(_lib.FilterDev)
    assert got[("size", "ScaoPlanDev")] == ctypes.sizeof(_lib.PlanDev)
    for f in fields_plan:
        assert got[("plan", f)] == getattr(_lib.PlanDev, f).offset, f
    for f in fields_filt:
        assert got[("filt", f)] == getattr(_lib.FilterDev, f).offset, f
    for f in _lib.FILTER_PARAM_DT.names:
        assert got[("fparam", f)] == _lib.FILTER_PARAM_DT.fields[f][1], f


def test_cpp_consumer_compiles_against_header():
    """The C++ host of tests/cabi (no Python, no torch) compiles against
    include/scao_b200.h and links against the library; it runs on a GPU in
    test_gpu_cabi_cpp.py."""
    import shutil
    import subprocess
    import tempfile
    cxx = shutil.which("g++")
    if cxx is None:
        import pytest
        pytest.skip("no host C++ compiler")
    cuda_inc = "/usr/local/cuda/include"
    lib = _lib.lib()._name
    with tempfile.TemporaryDirectory() as d:
        exe = os.path.join(d, "consumer")
        subprocess.check_call([cxx, "-std=c++17", "-O1", "-I", os.path.join(ROOT, "include"),
                               "-I", cuda_inc, os.path.join(ROOT, "tests", "cabi", "consumer.cpp"),
                               lib, "-L/usr/local/cuda/lib64", "-lcudart",
                               "-Wl,-rpath," + os.path.dirname(lib), "-o", exe])
        assert os.path.exists(exe)
