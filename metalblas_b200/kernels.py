"""Kernel library handle (the B200 counterpart of metalblas/kernels.py).

The reference compiles Metal source at run time (metalblas/kernels.py:55-57);
here every kernel is compiled ahead of time into ``libmetalblas_b200.so`` and
reached through the C ABI.  This module exposes the library and its probes.
"""
from __future__ import annotations

import ctypes

from . import _lib

library_path = _lib.LIB_PATH


def load():
    """Load the shared library (raises if it is missing and cannot be built)."""
    return _lib.load()


def has_tcgen05() -> bool:
    """True when the library was built for sm_100a and a CUDA device is present
    (the reference's has_metal4 probe, metalblas/kernels.py:65-73)."""
    import torch
    if not torch.cuda.is_available():
        return False
    major, minor = torch.cuda.get_device_capability()
    return _lib.load().mb_built_sm() == 100 and (major, minor) == (10, 0)


def plan(a, b, *, backend=None) -> str:
    """The plan mb_gemm would run for ``a @ b``: 2-D CUDA tensors, or 3-D
    batches as ``bmm`` takes them (a [B, M, K], b [B or 1, K, N], output
    row-major [B, M, N])."""
    from .dispatch import _BACKENDS, _matrix_view
    batched = a.dim() == 3
    M, K = a.shape[-2:]
    N = b.shape[-1]
    d = _lib.new_desc()
    d.dtype = _lib.DTYPE_CODE[a.dtype]
    d.backend = _BACKENDS[backend]
    d.M, d.N, d.K = M, N, K
    if batched:
        A, B = a, b
        d.batch = a.shape[0]
        d.a_rs, d.a_cs = A.stride()[1:]
        d.b_rs, d.b_cs = B.stride()[1:]
        d.sA = A.stride(0)
        d.sB = 0 if b.shape[0] == 1 else B.stride(0)
        d.sC = M * N
    else:
        A, B = _matrix_view(a, M, K), _matrix_view(b, K, N)
        d.a_rs, d.a_cs = A.stride()
        d.b_rs, d.b_cs = B.stride()
    d.A, d.B, d.C = A.data_ptr(), B.data_ptr(), A.data_ptr()
    d.c_rs, d.c_cs = N, 1
    d.workspace_bytes = -1  # plan as a call with a workspace (the public API always provides one)
    return _lib.plan_query(d)


def device_status() -> int:
    """0, or MB_ERR_DEVICE_TIMEOUT (4) when a bounded device wait gave up."""
    return _lib.device_status()


def device_status_clear() -> None:
    """Reset the status word and drop the cached split-K workspaces: a kernel that
    gave up may have left ticket counters non-zero, so fresh zeroed buffers are
    allocated on the next call."""
    from . import dispatch
    _lib.device_status_clear()
    dispatch.reset_caches()


def debug_wait_timeout(limit_us: int) -> None:
    """Launch a kernel whose wait can never complete; it must give up after
    ``limit_us`` microseconds and record MB_ERR_DEVICE_TIMEOUT."""
    import torch
    stream = torch.cuda.current_stream().cuda_stream
    _lib.raise_for(_lib.load().mb_debug_wait_timeout(int(limit_us), ctypes.c_void_p(stream)),
                   "mb_debug_wait_timeout")
