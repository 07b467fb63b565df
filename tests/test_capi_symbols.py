"""The C-ABI library loads without a GPU and exports every function include/trnopt_cuda.h declares, and the header
compiles as C99 and C++11. CPU only: no compute call is made here."""

import ctypes
import re

from conftest import ROOT


def declared_functions():
    text = (ROOT / "include" / "trnopt_cuda.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(trnopt_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_api():
    names = declared_functions()
    for must in ("trnopt_half_step", "trnopt_row_lse", "trnopt_workspace_size", "trnopt_median_cost"):
        assert must in names


def test_library_exports_every_declared_symbol():
    from trnopt import _capi
    lib = ctypes.CDLL(str(_capi.LIB_PATH))
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_every_declared_symbol():
    from trnopt import _capi
    assert sorted(_capi.exported_symbols()) == declared_functions()


def test_status_strings_without_gpu():
    from trnopt import _capi
    assert _capi.lib.trnopt_status_string(0) == b"ok"
    assert _capi.lib.trnopt_status_string(-3) == b"workspace missing or too small"
    assert _capi.lib.trnopt_version() >= 100


def test_header_compiles_as_c_and_cpp(tmp_path):
    """The header is usable from plain C (cgo, JNI glue, plugin hosts written in C) and from C++: every declared
    function is referenced through a function pointer, so a declaration that is not valid C fails here."""
    import shutil
    import subprocess
    import pytest
    names = declared_functions()
    body = "typedef void (*fn)(void);\nconst fn every[] = {\n" + "".join(f"  (fn){n},\n" for n in names) + "};\n"
    src = '#include "trnopt_cuda.h"\n' + body + "int main(void) { return (int)(sizeof every / sizeof every[0]) > 0 ? 0 : 1; }\n"
    inc = str(ROOT / "include")
    for compiler, ext, std in (("gcc", "c", "-std=c99"), ("g++", "cpp", "-std=c++11")):
        if shutil.which(compiler) is None:
            pytest.skip(f"{compiler} not installed")
        f = tmp_path / f"use.{ext}"
        f.write_text(src)
        r = subprocess.run([compiler, std, "-Wall", "-Wextra", "-Werror", "-pedantic", "-I", inc, "-c", str(f), "-o",
                            str(tmp_path / f"use_{ext}.o")], capture_output=True, text=True)
        assert r.returncode == 0, r.stderr
