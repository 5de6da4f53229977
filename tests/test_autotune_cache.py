"""CPU: the library's per-shape plan-override table (the autotune cache) and
mb_gemv's argument checks.  The planner runs in query mode here (no GPU), so
the tests read the plan text; nothing is launched."""
from __future__ import annotations

import ctypes
import os
import subprocess

import pytest
import torch

from metalblas_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _desc(M, N, K, dtype=torch.bfloat16):
    d = _lib.new_desc()
    d.dtype = _lib.DTYPE_CODE[dtype]
    d.M, d.N, d.K = M, N, K
    d.A = d.B = d.C = 1 << 20
    d.a_rs, d.a_cs = K, 1
    d.b_rs, d.b_cs = N, 1
    d.c_rs, d.c_cs = N, 1
    d.workspace_bytes = -1
    return d


@pytest.fixture
def clean_table(lib):
    lib.mb_autotune_cache_clear()
    yield lib
    lib.mb_autotune_cache_clear()


def test_override_layout_matches_c(tmp_path):
    fields = [f[0] for f in _lib.PlanOverride._fields_]
    prog = tmp_path / "ov.c"
    body = "\n".join(f'printf("{f} %zu\\n", offsetof(mb_plan_override, {f}));' for f in fields)
    prog.write_text(f'#include <stdio.h>\n#include <stddef.h>\n#include "metalblas_b200.h"\n'
                    f'int main(void){{ {body} printf("sizeof %zu\\n", sizeof(mb_plan_override)); return 0; }}\n')
    exe = tmp_path / "ov"
    subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), str(prog), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split("\n")
    got = dict(line.split() for line in out if line)
    for f in fields:
        assert int(got[f]) == getattr(_lib.PlanOverride, f).offset, f
    assert int(got["sizeof"]) == ctypes.sizeof(_lib.PlanOverride)


def test_record_lookup_and_plan(clean_table):
    d = _desc(2048, 2048, 4096)
    table_plan = _lib.plan_query(d)
    assert _lib.autotune_lookup(d) is None
    _lib.autotune_record(d, (_lib.MB_BACKEND_TC, 64, 2, -1))
    assert _lib.autotune_lookup(d) == (_lib.MB_BACKEND_TC, 64, 2, -1)
    assert clean_table.mb_autotune_cache_size() == 1
    # mb_gemm (and the plan query) now run the recorded plan for this shape ...
    tuned = _lib.plan_query(d)
    assert "bn=64" in tuned and "split=2" in tuned, tuned
    # ... but not for a descriptor that carries its own override
    q = _desc(2048, 2048, 4096)
    q.tile_n = 128
    assert "bn=128" in _lib.plan_query(q)
    # other shapes and layouts are separate keys
    assert _lib.autotune_lookup(_desc(2048, 2048, 2048)) is None
    t = _desc(2048, 2048, 4096)
    t.a_rs, t.a_cs = 1, 2048
    assert _lib.autotune_lookup(t) is None
    # "keep" records a tuned shape whose table plan stands
    _lib.autotune_record(d, None)
    assert _lib.autotune_lookup(d) == "keep"
    assert _lib.plan_query(d) == table_plan


def test_save_load_roundtrip(clean_table, tmp_path):
    path = str(tmp_path / "tune.txt")
    d1, d2 = _desc(4096, 4096, 4096), _desc(128, 8192, 65536)
    _lib.autotune_record(d1, (_lib.MB_BACKEND_TC, 128, 1, -1))
    _lib.autotune_record(d2, None)
    assert clean_table.mb_autotune_cache_save(path.encode()) == _lib.MB_OK
    assert not os.path.exists(path + ".tmp")
    clean_table.mb_autotune_cache_clear()
    assert clean_table.mb_autotune_cache_size() == 0
    assert clean_table.mb_autotune_cache_load(path.encode()) == _lib.MB_OK
    assert _lib.autotune_lookup(d1) == (_lib.MB_BACKEND_TC, 128, 1, -1)
    assert _lib.autotune_lookup(d2) == "keep"


def test_bad_files_change_nothing(clean_table, tmp_path):
    d = _desc(1024, 1024, 1024)
    _lib.autotune_record(d, (_lib.MB_BACKEND_TC, 32, 0, -1))
    missing = str(tmp_path / "nope.txt")
    assert clean_table.mb_autotune_cache_load(missing.encode()) == _lib.MB_ERR_INVALID
    bad = tmp_path / "bad.txt"
    bad.write_text("not an autotune file\nx\t1 2 3\n")
    assert clean_table.mb_autotune_cache_load(str(bad).encode()) == _lib.MB_ERR_INVALID
    good_header = tmp_path / "trunc.txt"
    good_header.write_text("metalblas_b200 autotune v1\nkey\t1 2\n")
    assert clean_table.mb_autotune_cache_load(str(good_header).encode()) == _lib.MB_ERR_INVALID
    assert clean_table.mb_autotune_cache_size() == 1
    assert _lib.autotune_lookup(d) == (_lib.MB_BACKEND_TC, 32, 0, -1)


def test_gemv_rejects_bad_arguments(lib):
    V = ctypes.c_void_p
    args = dict(dtype=_lib.MB_BF16, rows=4, cols=8, ldw=8, incx=1, incy=1)

    def call(**kw):
        a = dict(args, **kw)
        return lib.mb_gemv(a["dtype"], a.get("trans", 0), a["rows"], a["cols"], V(1 << 20), a["ldw"], V(1 << 20),
                           a["incx"], V(1 << 20), a["incy"], None, 0, None)

    assert call(trans=2) == _lib.MB_ERR_INVALID
    assert call(rows=-1) == _lib.MB_ERR_INVALID
    assert call(ldw=4) == _lib.MB_ERR_INVALID
    assert call(dtype=42) == _lib.MB_ERR_UNSUPPORTED


def test_tile_choice_memo_follows_alignment_and_strides():
    """The planner memoises its tile choice per thread; a descriptor that
    differs only in operand alignment or strides must get its own plan, and the
    first descriptor its original plan back afterwards."""
    d = _desc(2048, 2048, 2048)
    aligned = _lib.plan_query(d)
    assert aligned.startswith("tc ") and "a_mn=0" in aligned, aligned
    d.A = (1 << 20) + 2  # not 16-byte aligned: TMA cannot read A in place
    assert _lib.plan_query(d).startswith("tc_packed"), _lib.plan_query(d)
    d.A = 1 << 20
    assert _lib.plan_query(d) == aligned
    d.a_rs, d.a_cs = 1, 2048  # column-major A: MN-major tiles
    assert "a_mn=1" in _lib.plan_query(d), _lib.plan_query(d)
    d.a_rs, d.a_cs = 2048, 1
    assert _lib.plan_query(d) == aligned


def test_routing_of_wide_integers_complex64_and_thin_fp32():
    """The planner's routing rules, read from its plan text (no GPU): 16/32/64-bit
    integers go to byte planes on the int8 tensor cores (in exact K chunks),
    tiny ones stay on IMAD; complex64 runs as one real 3xTF32 GEMM unless a
    complex alpha needs the complex epilogue; thin fp32 products take the
    several-row column GEMV."""
    assert _lib.plan_query(_desc(2048, 2048, 2048, torch.int32)).startswith("tc_int_planes planes=4")
    assert _lib.plan_query(_desc(2048, 2048, 2048, torch.int16)).startswith("tc_int_planes planes=2")
    assert "chunks=2" in _lib.plan_query(_desc(130, 70, 5000, torch.int64))
    assert _lib.plan_query(_desc(64, 64, 64, torch.int32)) == "simt"
    c = _desc(4096, 4096, 4096, torch.complex64)
    assert _lib.plan_query(c).startswith("tc_c64x3"), _lib.plan_query(c)
    c.epilogue, c.alpha_nz, c.beta_nz, c.alpha_re, c.alpha_im = 1, 1, 0, 2.0, 1.0  # complex alpha, no bias
    assert _lib.plan_query(c) == "simt"
    c.alpha_im = 0.0  # a real alpha keeps the tensor cores
    assert _lib.plan_query(c).startswith("tc_c64x3")
    assert "rows=4" in _lib.plan_query(_desc(4, 14336, 4096, torch.float32))
    # the column GEMV fills whole waves of resident CTAs: 112 column blocks x 5 splits
    assert _lib.plan_query(_desc(1, 28672, 16384)) == "gemv_cols vec=8 ksplit=5"
