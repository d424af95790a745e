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
