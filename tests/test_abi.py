"""CPU: the C-ABI library loads and exports every symbol include/faie2fn.h declares (no compute without a GPU)."""

import ctypes
import os
import re

from fn import EXPORTS, FN

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions():
    txt = open(os.path.join(ROOT, "include", "faie2fn.h")).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(fn_\w+)\s*\(", txt)))


def test_header_declares_the_ctypes_surface():
    assert sorted(EXPORTS) == header_functions()


def test_library_exports_every_declared_symbol(libpath):
    lib = ctypes.CDLL(libpath)
    missing = [s for s in header_functions() if not hasattr(lib, s)]
    assert not missing, missing


def test_library_hides_internal_symbols(libpath):
    # only the fn_* C ABI is exported (built with -fvisibility=hidden)
    import subprocess
    out = subprocess.run(["nm", "-D", "--defined-only", libpath], capture_output=True, text=True).stdout
    names = [l.split()[-1] for l in out.splitlines() if " T " in l]
    assert names and all(n.startswith("fn_") for n in names), [n for n in names if not n.startswith("fn_")][:10]


def test_fn_class_binds_and_reports_errors_without_gpu(libpath):
    f = FN(libpath)
    # an unsupported type id fails cleanly before any device work
    rc = f.d.fn_gemv_plan(99, 16, 256, __import__("numpy").zeros(7, "int32"))
    assert rc == -1
    assert f.d.fn_error().decode()
