"""ctypes binding of the C ABI in ``include/metalblas_b200.h``.

The shared library is the product: there is no Python or CPU fallback.  If the
library is missing, or the tensors are not on a CUDA device, every entry point
raises.  ``load()`` builds the library in-tree when it is absent and nvcc is
available (the development container); on a GPU box the prebuilt in-tree
``libmetalblas_b200.so`` is used.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libmetalblas_b200.so")

# mb_dtype
MB_F32, MB_F16, MB_BF16, MB_C64, MB_C32, MB_I8, MB_U8, MB_I16, MB_I32, MB_I64 = range(10)
# mb_backend
MB_BACKEND_AUTO, MB_BACKEND_GEMV, MB_BACKEND_TC, MB_BACKEND_SIMT = range(4)
# mb_status
MB_OK, MB_ERR_INVALID, MB_ERR_UNSUPPORTED, MB_ERR_LAUNCH, MB_ERR_DEVICE_TIMEOUT, MB_ERR_WORKSPACE = range(6)

DTYPE_CODE = {
    torch.float32: MB_F32, torch.float16: MB_F16, torch.bfloat16: MB_BF16,
    torch.complex64: MB_C64, torch.complex32: MB_C32,
    torch.int8: MB_I8, torch.uint8: MB_U8, torch.int16: MB_I16,
    torch.int32: MB_I32, torch.int64: MB_I64,
}

# Every symbol the header declares (checked by the CPU test suite).
EXPORTS = (
    "mb_gemm_desc_init", "mb_gemm", "mb_gemm_noalloc", "mb_gemm_workspace_size", "mb_plan_query",
    "mb_last_error_string", "mb_device_status", "mb_device_status_clear",
    "mb_debug_wait_timeout", "mb_abi_version", "mb_built_sm", "mb_gemv",
    "mb_autotune_record", "mb_autotune_lookup", "mb_autotune_cache_load", "mb_autotune_cache_save",
    "mb_autotune_cache_clear", "mb_autotune_cache_size", "mb_peak_probe",
    "mb_gemm_peer", "mb_ipc_get_handle", "mb_ipc_open", "mb_ipc_close",
)

MB_MAX_PEERS = 7


class GemmDesc(ctypes.Structure):
    """Mirror of ``mb_gemm_desc`` (field order and C types must match)."""

    _fields_ = [
        ("dtype", ctypes.c_int32), ("backend", ctypes.c_int32),
        ("M", ctypes.c_int64), ("N", ctypes.c_int64), ("K", ctypes.c_int64), ("batch", ctypes.c_int64),
        ("A", ctypes.c_void_p), ("B", ctypes.c_void_p), ("C", ctypes.c_void_p),
        ("a_rs", ctypes.c_int64), ("a_cs", ctypes.c_int64), ("sA", ctypes.c_int64),
        ("b_rs", ctypes.c_int64), ("b_cs", ctypes.c_int64), ("sB", ctypes.c_int64),
        ("c_rs", ctypes.c_int64), ("c_cs", ctypes.c_int64), ("sC", ctypes.c_int64),
        ("conj_a", ctypes.c_int32), ("conj_b", ctypes.c_int32),
        ("epilogue", ctypes.c_int32), ("alpha_nz", ctypes.c_int32), ("beta_nz", ctypes.c_int32),
        ("stream_k", ctypes.c_int32),
        ("bias", ctypes.c_void_p),
        ("bias_rs", ctypes.c_int64), ("bias_cs", ctypes.c_int64), ("bias_bs", ctypes.c_int64),
        ("alpha_re", ctypes.c_double), ("alpha_im", ctypes.c_double),
        ("beta_re", ctypes.c_double), ("beta_im", ctypes.c_double),
        ("ialpha", ctypes.c_int64), ("ibeta", ctypes.c_int64),
        ("tile_n", ctypes.c_int32), ("split_k", ctypes.c_int32), ("swap_ab", ctypes.c_int32),
        ("cta_pair", ctypes.c_int32),
        ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_int64),
    ]


class PeerTargets(ctypes.Structure):
    """Mirror of ``mb_peer_targets``."""

    _fields_ = [("count", ctypes.c_int32), ("C", ctypes.c_void_p * MB_MAX_PEERS), ("mc_C", ctypes.c_void_p)]


def peer_targets(addrs, mc=None) -> PeerTargets:
    """An mb_peer_targets holding the given device addresses (and the
    multicast address of C, if any)."""
    addrs = list(addrs)
    if len(addrs) > MB_MAX_PEERS:
        raise ValueError(f"at most {MB_MAX_PEERS} peers, got {len(addrs)}")
    t = PeerTargets()
    t.count = len(addrs)
    for i, a in enumerate(addrs):
        t.C[i] = int(a)
    t.mc_C = int(mc) if mc else None
    return t


class PlanOverride(ctypes.Structure):
    """Mirror of ``mb_plan_override``."""

    _fields_ = [(n, ctypes.c_int32) for n in
                ("keep", "backend", "tile_n", "split_k", "swap_ab", "cta_pair", "stream_k")]


_lib = None
_lock = threading.Lock()


def load():
    """Load (building first if needed and possible) the shared library."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            from . import build as _build
            _build.build()
        lib = ctypes.CDLL(LIB_PATH)
        P = ctypes.POINTER(GemmDesc)
        lib.mb_gemm_desc_init.argtypes = [P]
        lib.mb_gemm_desc_init.restype = None
        lib.mb_gemm.argtypes = [P, ctypes.c_void_p]
        lib.mb_gemm.restype = ctypes.c_int
        lib.mb_gemm_noalloc.argtypes = [P, ctypes.c_void_p]
        lib.mb_gemm_noalloc.restype = ctypes.c_int
        lib.mb_gemm_workspace_size.argtypes = [P]
        lib.mb_gemm_workspace_size.restype = ctypes.c_int64
        lib.mb_plan_query.argtypes = [P, ctypes.c_char_p, ctypes.c_int]
        lib.mb_plan_query.restype = ctypes.c_int
        lib.mb_last_error_string.argtypes = []
        lib.mb_last_error_string.restype = ctypes.c_char_p
        lib.mb_device_status.argtypes = []
        lib.mb_device_status.restype = ctypes.c_int
        lib.mb_device_status_clear.argtypes = []
        lib.mb_device_status_clear.restype = None
        lib.mb_debug_wait_timeout.argtypes = [ctypes.c_int64, ctypes.c_void_p]
        lib.mb_debug_wait_timeout.restype = ctypes.c_int
        lib.mb_abi_version.argtypes = []
        lib.mb_abi_version.restype = ctypes.c_int
        lib.mb_built_sm.argtypes = []
        lib.mb_built_sm.restype = ctypes.c_int
        V, I64, I32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32
        lib.mb_gemv.argtypes = [I32, I32, I64, I64, V, I64, V, I64, V, I64, V, I64, V]
        lib.mb_gemv.restype = ctypes.c_int
        PO = ctypes.POINTER(PlanOverride)
        lib.mb_autotune_record.argtypes = [P, PO]
        lib.mb_autotune_record.restype = ctypes.c_int
        lib.mb_autotune_lookup.argtypes = [P, PO]
        lib.mb_autotune_lookup.restype = ctypes.c_int
        lib.mb_autotune_cache_load.argtypes = [ctypes.c_char_p]
        lib.mb_autotune_cache_load.restype = ctypes.c_int
        lib.mb_autotune_cache_save.argtypes = [ctypes.c_char_p]
        lib.mb_autotune_cache_save.restype = ctypes.c_int
        lib.mb_autotune_cache_clear.argtypes = []
        lib.mb_autotune_cache_clear.restype = None
        lib.mb_autotune_cache_size.argtypes = []
        lib.mb_autotune_cache_size.restype = ctypes.c_int64
        lib.mb_peak_probe.argtypes = [I32, ctypes.POINTER(ctypes.c_double)]
        lib.mb_peak_probe.restype = ctypes.c_int
        lib.mb_gemm_peer.argtypes = [P, ctypes.POINTER(PeerTargets), V]
        lib.mb_gemm_peer.restype = ctypes.c_int
        lib.mb_ipc_get_handle.argtypes = [V, V, ctypes.POINTER(I64)]
        lib.mb_ipc_get_handle.restype = ctypes.c_int
        lib.mb_ipc_open.argtypes = [V, ctypes.POINTER(V)]
        lib.mb_ipc_open.restype = ctypes.c_int
        lib.mb_ipc_close.argtypes = [V]
        lib.mb_ipc_close.restype = ctypes.c_int
        _lib = lib
        return lib


_fast = None
_fast_tried = False


def fast():
    """The host fast path (csrc/fastpath.cpp, built in tree as _mbfast*.so) with
    this library's mb_gemm registered, or None when it is not built.  Without
    it every call takes the Python path; the products are the same."""
    global _fast, _fast_tried
    if _fast_tried:
        return _fast
    lib = load()  # before taking the lock: load() takes it too
    with _lock:
        if _fast_tried:
            return _fast
        import importlib.util
        import sysconfig
        path = os.path.join(_PKG, "_mbfast" + sysconfig.get_config_var("EXT_SUFFIX"))
        mod = None
        if os.path.exists(path):
            spec = importlib.util.spec_from_file_location("_mbfast", path)
            mod = importlib.util.module_from_spec(spec)
            spec.loader.exec_module(mod)
            if mod.desc_size() != ctypes.sizeof(GemmDesc):
                raise RuntimeError("_mbfast was built against a different mb_gemm_desc; rebuild the package")
            fn = ctypes.cast(lib.mb_gemm, ctypes.c_void_p).value
            mod.set_gemm(fn)
        _fast = mod
        _fast_tried = True
        return _fast


def last_error() -> str:
    return load().mb_last_error_string().decode(errors="replace")


def raise_for(code: int, what: str = "mb_gemm") -> None:
    """Map an mb_status onto the reference's exception types."""
    if code == MB_OK:
        return
    msg = f"{what}: {last_error()}"
    if code == MB_ERR_INVALID:
        raise ValueError(msg)
    if code == MB_ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    if code == MB_ERR_WORKSPACE:
        raise ValueError(msg)
    raise RuntimeError(msg)


def new_desc() -> GemmDesc:
    d = GemmDesc()
    load().mb_gemm_desc_init(ctypes.byref(d))
    return d


def plan_query(d: GemmDesc) -> str:
    buf = ctypes.create_string_buffer(256)
    n = load().mb_plan_query(ctypes.byref(d), buf, 256)
    if n < 0:
        raise_for(-n, "mb_plan_query")
    return buf.value.decode()


def device_status() -> int:
    return int(load().mb_device_status())


def device_status_clear() -> None:
    load().mb_device_status_clear()


def autotune_lookup(d: GemmDesc):
    """The library's cached plan override for d's shape: None on a miss, "keep"
    when tuning kept the tile table's choice, else (backend, tile_n, split_k,
    swap_ab)."""
    ov = PlanOverride()
    rc = load().mb_autotune_lookup(ctypes.byref(d), ctypes.byref(ov))
    if rc < 0:
        raise_for(-rc, "mb_autotune_lookup")
    if rc == 0:
        return None
    if ov.keep:
        return "keep"
    return (ov.backend, ov.tile_n, ov.split_k, ov.swap_ab)


def autotune_record(d: GemmDesc, choice) -> None:
    """Record choice (None = keep the table's plan) for d's shape."""
    ov = PlanOverride()
    if choice is None:
        ov.keep = 1
    else:
        ov.backend, ov.tile_n, ov.split_k, ov.swap_ab = (int(x) for x in choice)
    raise_for(load().mb_autotune_record(ctypes.byref(d), ctypes.byref(ov)), "mb_autotune_record")


def peak_probe(kind: int) -> float:
    """Measured CUDA-core multiply-add rate in 1e12 ops/s (0 fp32, 1 int32, 2 int64)."""
    v = ctypes.c_double()
    raise_for(load().mb_peak_probe(int(kind), ctypes.byref(v)), "mb_peak_probe")
    return v.value
