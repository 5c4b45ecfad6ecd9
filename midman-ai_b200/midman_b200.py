"""ctypes binding of libmidman_gpu.so (include/midman_gpu.h, include/midman_api.h).

This is how Python callers (the tests and bench.py) reach the library: the same
C ABI a Rust FFI crate or a C program binds. Loading fails loudly when the
shared library is missing; there is no fallback implementation.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "lib" / "libmidman_gpu.so"

# Every symbol the public headers declare, grouped by header.
GPU_SYMBOLS = [
    "mm_gpu_last_error", "mm_gpu_device_status", "mm_gpu_gemm",
]
API_SYMBOLS: list[str] = []

_lib = None


def _sig(lib, name, restype, *argtypes):
    f = getattr(lib, name)
    f.restype = restype
    f.argtypes = list(argtypes)


def load(path: str | os.PathLike | None = None) -> C.CDLL:
    """Loads (once) and returns the library with every signature declared."""
    global _lib
    if _lib is not None:
        return _lib
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise FileNotFoundError(f"{p} is missing: run `python midman-ai_b200/build.py` first")
    lib = C.CDLL(str(p))
    i32, i64, f32p, vp = C.c_int32, C.c_int64, C.POINTER(C.c_float), C.c_void_p
    _sig(lib, "mm_gpu_last_error", C.c_char_p)
    _sig(lib, "mm_gpu_device_status", i32, vp)
    _sig(lib, "mm_gpu_gemm", i32, i32, i32, i32, vp, i64, i32, vp, i64, i32, vp, i64, vp, i64, i32, vp)
    _lib = lib
    return lib


class MidmanGpuError(RuntimeError):
    pass


def check(rc: int) -> int:
    if rc < 0:
        msg = load().mm_gpu_last_error().decode(errors="replace")
        raise MidmanGpuError(f"status {rc}: {msg}")
    return rc


def _ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(stream) -> int | None:
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    return stream


def gemm(a, b, c, *, m, n, k, lda, ldb, ldc, a_mn_major, b_mn_major, r=None, ldr=0,
         precision=0, stream=None):
    """C = A(m,k) B(n,k)^T (+R) on torch CUDA tensors (see include/midman_gpu.h)."""
    return check(load().mm_gpu_gemm(m, n, k, _ptr(a), lda, int(a_mn_major), _ptr(b), ldb,
                                    int(b_mn_major), _ptr(c), ldc, _ptr(r), ldr, precision,
                                    _stream(stream)))


def device_status(stream=None):
    return check(load().mm_gpu_device_status(_stream(stream)))
