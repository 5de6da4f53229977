"""CPU: the C-ABI library loads, exports every symbol include/metalblas_b200.h
declares, and the ctypes mirror of mb_gemm_desc has the C layout.  No compute
call is made (there is no GPU here)."""
from __future__ import annotations

import ctypes
import os
import re
import subprocess

import pytest

from metalblas_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "metalblas_b200.h")


def header_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(mb_[a-z_0-9]+)\s*\(", src)))


def test_header_lists_match_binding():
    assert header_functions() == sorted(_lib.EXPORTS)


def test_library_exports_every_declared_symbol(lib):
    for name in header_functions():
        assert hasattr(lib, name), f"{name} not exported"


def test_library_is_sm100a(lib):
    assert lib.mb_built_sm() == 100
    assert lib.mb_abi_version() == 1


def test_desc_init_defaults(lib):
    d = _lib.new_desc()
    assert d.batch == 1 and d.alpha_re == 1.0 and d.beta_re == 1.0
    assert d.ialpha == 1 and d.ibeta == 1 and d.backend == _lib.MB_BACKEND_AUTO and d.epilogue == 0


def test_desc_layout_matches_c(tmp_path):
    fields = [f[0] for f in _lib.GemmDesc._fields_]
    prog = tmp_path / "off.c"
    body = "\n".join(f'printf("{f} %zu\\n", offsetof(mb_gemm_desc, {f}));' for f in fields)
    prog.write_text(f'#include <stdio.h>\n#include <stddef.h>\n#include "metalblas_b200.h"\n'
                    f'int main(void){{ {body} printf("sizeof %zu\\n", sizeof(mb_gemm_desc)); return 0; }}\n')
    exe = tmp_path / "off"
    subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), str(prog), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split("\n")
    got = dict(line.split() for line in out if line)
    for f in fields:
        assert int(got[f]) == getattr(_lib.GemmDesc, f).offset, f
    assert int(got["sizeof"]) == ctypes.sizeof(_lib.GemmDesc)


def test_error_string_is_text(lib):
    assert isinstance(_lib.last_error(), str)


def test_status_codes_map_to_reference_exceptions():
    with pytest.raises(ValueError):
        _lib.raise_for(_lib.MB_ERR_INVALID)
    with pytest.raises(NotImplementedError):
        _lib.raise_for(_lib.MB_ERR_UNSUPPORTED)
    with pytest.raises(RuntimeError):
        _lib.raise_for(_lib.MB_ERR_DEVICE_TIMEOUT)
    _lib.raise_for(_lib.MB_OK)


def test_fast_path_extension_matches_the_descriptor_layout(lib):
    """The host fast path (csrc/fastpath.cpp) is built in tree and was compiled
    against this header's mb_gemm_desc."""
    from metalblas_b200 import _lib as L
    fast = L.fast()
    assert fast is not None, "the _mbfast extension is not built"
    assert fast.desc_size() == ctypes.sizeof(L.GemmDesc)
