"""CPU: the C-ABI library builds, loads, and exports every symbol include/cvhrf.h declares."""
import ctypes
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    src = open(os.path.join(ROOT, "include", "cvhrf.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(cvhrf_\w+)\s*\(", src)))


def test_library_exports_all_declared_symbols():
    from complex_valued_holographic_radiance_fields_b200 import _lib
    L = _lib.lib()
    names = declared_functions()
    assert len(names) >= 12
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing
    assert set(names) <= set(_lib.SIGNATURES), set(names) - set(_lib.SIGNATURES)


def test_status_strings_and_size_queries():
    from complex_valued_holographic_radiance_fields_b200 import _lib
    L = _lib.lib()
    assert L.cvhrf_status_string(0) == b"ok"
    assert L.cvhrf_version() >= 100
    assert L.cvhrf_asm_workspace_bytes(800, 9, 800, 800, 3, 800, 800) >= 9 * 800 * 1600 * 8
    assert L.cvhrf_raster_geometry_workspace_bytes(300000, 3, 3) > 300000 * 64
    assert L.cvhrf_raster_backward_workspace_bytes(1000, 3, 3) >= 1000 * 15 * 4


def test_invalid_arguments_rejected_without_gpu():
    from complex_valued_holographic_radiance_fields_b200 import _lib
    L = _lib.lib()
    plan = ctypes.c_void_p()
    assert L.cvhrf_asm_plan_create(7, ctypes.byref(plan)) != 0      # too small
    assert L.cvhrf_asm_plan_create(8 * 7, ctypes.byref(plan)) != 0  # factor 7 unsupported
    assert L.cvhrf_sparse_adam(None, 1, None, 0, 0.9, 0.999, None) == 1
