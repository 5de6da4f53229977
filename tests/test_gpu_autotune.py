"""GPU: the autotuner (METALBLAS_AUTOTUNE) records its verdicts in the library's
plan-override table, persists them through METALBLAS_AUTOTUNE_CACHE, and a
tuned plan gives the oracle's answer; mb_gemv through the C ABI."""
from __future__ import annotations

import ctypes

import pytest
import torch

import metalblas_b200 as mb
from metalblas_b200 import _lib, plan
from oracle import oracle as orc
from tests.helpers import NAME, rand, to_np

pytestmark = pytest.mark.gpu


@pytest.fixture
def tuner(monkeypatch, tmp_path):
    path = tmp_path / "tune.txt"
    monkeypatch.setattr(plan, "AUTOTUNE", True)
    monkeypatch.setenv("METALBLAS_AUTOTUNE_CACHE", str(path))
    plan.clear()
    monkeypatch.setattr(plan, "_loaded", False)
    yield path
    plan.clear()
    monkeypatch.setattr(plan, "_loaded", False)


@pytest.mark.parametrize("shape", [(2048, 2048, 2048), (128, 4096, 16384)])
def test_tuned_plans_match_oracle_and_persist(tuner, shape):
    M, N, K = shape
    gen = torch.Generator().manual_seed(12)
    a = rand((M, K), torch.bfloat16, gen)
    b = rand((K, N), torch.bfloat16, gen)
    ref = orc.product(to_np(a), to_np(b), "bfloat16")
    lib = _lib.load()
    assert lib.mb_autotune_cache_size() == 0
    for _ in range(2):  # the first call tunes, the second reuses the verdict
        ok, err = orc.check(to_np(mb.matmul(a, b)), ref, "bfloat16")
        assert ok, f"{shape} err={err}"
    assert lib.mb_autotune_cache_size() == 1
    assert tuner.exists() and tuner.read_text().startswith("metalblas_b200 autotune v1")
    # a fresh table loads the verdict from the file
    plan.clear()
    assert lib.mb_autotune_cache_load(str(tuner).encode()) == _lib.MB_OK
    assert lib.mb_autotune_cache_size() == 1
    ok, err = orc.check(to_np(mb.matmul(a, b)), ref, "bfloat16")
    assert ok, f"{shape} after reload err={err}"
    assert mb.kernels.device_status() == 0


def _gemv(W, x, y, trans, ws=None):
    lib = _lib.load()
    rows, cols = W.shape
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.mb_gemv(_lib.DTYPE_CODE[W.dtype], trans, rows, cols, W.data_ptr(), W.stride(0), x.data_ptr(),
                     x.stride(0), y.data_ptr(), y.stride(0), ws.data_ptr() if ws is not None else None,
                     ws.numel() if ws is not None else 0, ctypes.c_void_p(stream))
    _lib.raise_for(rc, "mb_gemv")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32, torch.int32, torch.complex64], ids=NAME.get)
def test_mb_gemv_both_orientations(dtype):
    gen = torch.Generator().manual_seed(13)
    rows, cols = 3000, 5000
    W = rand((rows, cols), dtype, gen)
    ws = torch.zeros(64 << 20, dtype=torch.uint8, device="cuda")
    for trans in (0, 1):
        n_in, n_out = (cols, rows) if trans == 0 else (rows, cols)
        for inc in (1, 3):
            xs = rand((n_in * inc,), dtype, gen)
            x = xs[::inc]
            ybuf = torch.zeros(n_out * 2, dtype=dtype, device="cuda")
            y = ybuf[::2]
            Wn, xn = to_np(W), to_np(x)
            if trans == 0:
                ref = orc.product(Wn, xn[:, None], NAME[dtype])[:, 0]
            else:
                ref = orc.product(xn[None, :], Wn, NAME[dtype])[0]
            for w in (None, ws):
                ybuf.zero_()
                _gemv(W, x, y, trans, w)
                ok, err = orc.check(to_np(y), ref, NAME[dtype])
                assert ok, f"trans={trans} inc={inc} ws={w is not None} err={err}"
                assert not to_np(ybuf[1::2]).any(), "wrote between strided outputs"


def test_peak_probe_rates_are_plausible():
    """The CUDA-core roofline denominators: B200 fp32 FFMA is 148 SMs x 128
    lanes x 2 ops x ~1.9 GHz ~ 72e12 op/s nominal; IMAD and the emulated int64
    multiply-add are slower."""
    f32 = _lib.peak_probe(0)
    i32 = _lib.peak_probe(1)
    i64 = _lib.peak_probe(2)
    assert 30.0 < f32 < 120.0, f32
    assert 5.0 < i32 <= f32 * 1.05, i32
    assert 0.5 < i64 < i32, i64
