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
    "mm_gpu_last_error", "mm_gpu_device_status", "mm_gpu_gemm", "mm_gpu_gemm_sum", "mm_gpu_clip_adamw", "mm_gpu_attention_forward",
    "mm_gpu_attention_backward", "mm_gpu_attention_forward_noalloc", "mm_gpu_rmsnorm_forward",
    "mm_gpu_rmsnorm_backward", "mm_gpu_rope", "mm_gpu_swiglu_forward", "mm_gpu_swiglu_backward",
    "mm_gpu_embedding_forward", "mm_gpu_embedding_backward", "mm_gpu_cross_entropy", "mm_gpu_comm_create",
    "mm_gpu_comm_destroy", "mm_gpu_allreduce_bucket", "mm_gpu_comm_wait", "mm_gpu_wait_selftest",
]
TENSOR_SYMBOLS = [
    "mm_tape_create", "mm_tape_destroy", "mm_tensor_new", "mm_tensor_shape", "mm_tensor_read", "mm_tensor_grad",
    "mm_tensor_free", "mm_tape_backward", "mm_op_matmul", "mm_op_add", "mm_op_mul", "mm_op_embedding",
    "mm_op_rms_norm", "mm_op_rope", "mm_op_causal_attention", "mm_op_swiglu", "mm_op_cross_entropy",
]
API_SYMBOLS = [
    "midman_abi_version", "midman_alloc", "midman_free", "midman_text_ptr", "midman_text_len",
    "midman_floats_ptr", "midman_floats_len", "midman_error_ptr", "midman_error_len", "midman_describe",
    "midman_preset_config", "midman_config_report", "midman_rope_table", "midman_lab_create",
    "midman_lab_step", "midman_lab_eval", "midman_lab_stats", "midman_lab_attention", "midman_lab_embedding",
    "midman_lab_destroy", "midman_nccl_unique_id", "midman_train_create", "midman_train_step",
    "midman_train_stage", "midman_train_step_staged", "midman_train_loss_and_grads", "midman_train_read",
    "midman_train_load", "midman_train_describe", "midman_train_eval", "midman_train_destroy",
    "midman_train_stream", "midman_train_profile", "midman_batcher_create", "midman_batcher_synthetic",
    "midman_batcher_next", "midman_batcher_destroy", "midman_train_save", "midman_train_restore",
    "midman_state_inspect", "midman_shard_inspect", "midman_batcher_open", "midman_batcher_seek", "midman_train_run",
    "midman_shard_read", "midman_shard_write", "midman_sha256", "midman_train_evaluate",
    "midman_train_shard_optimizer", "midman_shard_plan", "midman_train_params", "midman_train_grads",
]
STATUS = {0: "OK", 1: "STOPPED", -1: "ARGUMENT", -2: "CONFIG", -3: "SHAPE", -4: "INDEX", -5: "OTHER",
          -6: "DEVICE", -99: "PANIC"}

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
    _sig(lib, "mm_gpu_gemm_sum", i32, i32, i32, i32, C.POINTER(vp), C.POINTER(i64), i32, C.POINTER(vp),
         C.POINTER(i64), i32, C.POINTER(C.c_int32), vp, i64, vp, i64, vp)
    _sig(lib, "mm_gpu_clip_adamw", i32, i32, C.POINTER(i64), C.POINTER(C.c_int32), vp, vp, vp, vp, C.c_double,
         C.c_double, C.c_double, C.c_double, C.c_double, C.c_double, C.c_uint64, f32p, vp)
    _sig(lib, "mm_gpu_attention_forward", i32, i32, i32, i32, i32, i32, vp, vp, vp, i64, i64, vp, vp, i32, vp)
    _sig(lib, "mm_gpu_attention_backward", i32, i32, i32, i32, i32, i32, vp, vp, vp, vp, vp, vp, i64, i64, vp, vp,
         vp, i32, vp)
    _sig(lib, "mm_gpu_attention_forward_noalloc", i32, i32, i32, i32, i32, i32, vp, vp, vp, i64, i64, vp, vp, vp,
         vp)
    u32, u8p, dp, i32p = C.c_uint32, C.POINTER(C.c_uint8), C.POINTER(C.c_double), C.POINTER(C.c_int32)
    _sig(lib, "mm_gpu_rmsnorm_forward", i32, i32, i32, vp, vp, C.c_float, vp, vp, vp)
    _sig(lib, "mm_gpu_rmsnorm_backward", i32, i32, i32, vp, vp, vp, vp, vp, vp, vp, vp)
    _sig(lib, "mm_gpu_rope", i32, i32, i32, i32, i32, vp, i64, vp, vp, i32, vp)
    _sig(lib, "mm_gpu_swiglu_forward", i32, i64, vp, vp, vp, vp)
    _sig(lib, "mm_gpu_swiglu_backward", i32, i64, vp, vp, vp, vp)
    _sig(lib, "mm_gpu_embedding_forward", i32, i32, vp, i32, i32, vp, vp, vp)
    _sig(lib, "mm_gpu_embedding_backward", i32, i32, i32p, i32, i32, vp, vp, vp)
    _sig(lib, "mm_gpu_cross_entropy", i32, i32, i32, vp, i64, vp, C.c_float, vp, vp, vp)
    _sig(lib, "mm_gpu_comm_create", i32, u8p, i32, i32, C.POINTER(vp))
    _sig(lib, "mm_gpu_comm_destroy", i32, vp)
    _sig(lib, "mm_gpu_allreduce_bucket", i32, vp, vp, i64, i32, vp)
    _sig(lib, "mm_gpu_comm_wait", i32, vp, vp, i32)
    _sig(lib, "mm_gpu_wait_selftest", i32, i32, vp)
    u64, i64p = C.c_uint64, C.POINTER(C.c_int64)
    _sig(lib, "mm_tape_create", u32, i32)
    _sig(lib, "mm_tape_destroy", i32, u32)
    _sig(lib, "mm_tensor_new", u64, u32, i64p, i32, f32p, i32)
    _sig(lib, "mm_tensor_shape", i32, u32, u64, i64p, i32p)
    _sig(lib, "mm_tensor_read", i32, u32, u64, f32p, i64)
    _sig(lib, "mm_tensor_grad", i32, u32, u64, f32p, i64)
    _sig(lib, "mm_tensor_free", i32, u32, u64)
    _sig(lib, "mm_tape_backward", i32, u32, u64)
    _sig(lib, "mm_op_matmul", u64, u32, u64, u64, i32)
    _sig(lib, "mm_op_add", u64, u32, u64, u64)
    _sig(lib, "mm_op_mul", u64, u32, u64, u64)
    _sig(lib, "mm_op_embedding", u64, u32, u64, i32p, i64)
    _sig(lib, "mm_op_rms_norm", u64, u32, u64, u64, C.c_float)
    _sig(lib, "mm_op_rope", u64, u32, u64, i32, i32, C.c_float)
    _sig(lib, "mm_op_causal_attention", u64, u32, u64, u64, u64, i32, i32, i32, i32)
    _sig(lib, "mm_op_swiglu", u64, u32, u64, u64)
    _sig(lib, "mm_op_cross_entropy", u64, u32, u64, i32p, i64)
    _sig(lib, "midman_abi_version", u32)
    _sig(lib, "midman_alloc", u8p, u32)
    _sig(lib, "midman_free", None, u8p, u32)
    _sig(lib, "midman_text_ptr", u8p)
    _sig(lib, "midman_text_len", u32)
    _sig(lib, "midman_floats_ptr", f32p)
    _sig(lib, "midman_floats_len", u32)
    _sig(lib, "midman_error_ptr", u8p)
    _sig(lib, "midman_error_len", u32)
    _sig(lib, "midman_describe", i32)
    _sig(lib, "midman_preset_config", i32, u32, dp)
    _sig(lib, "midman_config_report", i32, dp)
    _sig(lib, "midman_rope_table", i32, u32, u32, C.c_double)
    _sig(lib, "midman_lab_create", u32, dp, dp, u32, u32, u32, u32)
    _sig(lib, "midman_lab_step", i32, u32, u32)
    _sig(lib, "midman_lab_eval", i32, u32)
    _sig(lib, "midman_lab_stats", i32, u32)
    _sig(lib, "midman_lab_attention", i32, u32, u32)
    _sig(lib, "midman_lab_embedding", i32, u32)
    _sig(lib, "midman_lab_destroy", i32, u32)
    _sig(lib, "midman_nccl_unique_id", i32, u8p)
    _sig(lib, "midman_train_create", u32, dp, dp, u32, u32, u32, u32, u32, u32, u32, u8p)
    _sig(lib, "midman_train_step", i32, u32, i32p, i32p)
    _sig(lib, "midman_train_stage", i32, u32, i32p, i32p)
    _sig(lib, "midman_train_step_staged", i32, u32, u32)
    _sig(lib, "midman_train_loss_and_grads", i32, u32, i32p, i32p)
    _sig(lib, "midman_train_read", i32, u32, u32, u32)
    _sig(lib, "midman_train_load", i32, u32, f32p, C.c_uint64)
    _sig(lib, "midman_train_describe", i32, u32)
    _sig(lib, "midman_train_eval", i32, u32, i32p, i32p, u32, u32)
    _sig(lib, "midman_train_destroy", i32, u32)
    _sig(lib, "midman_train_stream", i32, u32, C.POINTER(C.c_uint64))
    _sig(lib, "midman_train_profile", i32, u32, u32)
    _sig(lib, "midman_batcher_create", i32, C.POINTER(C.c_uint32), C.c_uint64, u32, u32, u32, u32, u32)
    _sig(lib, "midman_batcher_synthetic", i32, u32, u32, C.c_uint64, u32, u32, u32, u32)
    _sig(lib, "midman_batcher_next", i32, u32, i32p, i32p)
    _sig(lib, "midman_batcher_destroy", i32, u32)
    _sig(lib, "midman_train_save", i32, u32, u8p, u32, u32, u32, C.c_uint64, C.c_uint64)
    _sig(lib, "midman_train_restore", i32, u32, u8p, u32, u32, u32)
    _sig(lib, "midman_state_inspect", i32, u8p, u32)
    _sig(lib, "midman_shard_inspect", i32, u8p, u32)
    _sig(lib, "midman_batcher_open", i32, u8p, u32, u32, u32, u32, u32)
    _sig(lib, "midman_batcher_seek", i32, u32, C.c_uint64, C.c_uint64)
    _sig(lib, "midman_train_run", i32, u32, u32, u32)
    _sig(lib, "midman_shard_read", i32, u8p, u32, C.POINTER(C.c_uint32), C.c_uint64)
    _sig(lib, "midman_shard_write", i32, u8p, u32, u32, u32, C.POINTER(C.c_uint32), C.c_uint64)
    _sig(lib, "midman_sha256", i32, u8p, C.c_uint64, u8p)
    _sig(lib, "midman_train_evaluate", i32, u32, u8p, u32, C.c_uint64)
    _sig(lib, "midman_train_shard_optimizer", i32, u32, u32)
    _sig(lib, "midman_shard_plan", i32, dp, u32)
    _sig(lib, "midman_train_params", i32, u32, u32)
    _sig(lib, "midman_train_grads", i32, u32, u32)
    _lib = lib
    return lib


class MidmanGpuError(RuntimeError):
    def __init__(self, status, message):
        super().__init__(f"status {status}: {message}")
        self.status = status


def check(rc: int) -> int:
    if rc < 0:
        raise MidmanGpuError(rc, load().mm_gpu_last_error().decode(errors="replace"))
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


def gemm_sum(terms, c, *, m, n, ldc, a_mn_major, b_mn_major, r=None, ldr=0, stream=None):
    """C = sum of A_g(m,k_g) B_g(n,k_g)^T (+R); terms: [(a, lda, b, ldb, k), ...] (TF32)."""
    g = len(terms)
    a = (C.c_void_p * g)(*[_ptr(t[0]) for t in terms])
    lda = (C.c_int64 * g)(*[t[1] for t in terms])
    b = (C.c_void_p * g)(*[_ptr(t[2]) for t in terms])
    ldb = (C.c_int64 * g)(*[t[3] for t in terms])
    ks = (C.c_int32 * g)(*[t[4] for t in terms])
    return check(load().mm_gpu_gemm_sum(m, n, g, a, lda, int(a_mn_major), b, ldb, int(b_mn_major), ks, _ptr(c), ldc,
                                        _ptr(r), ldr, _stream(stream)))


def clip_adamw(p, g, m, v, numel, decay, *, max_norm, lr, beta1, beta2, eps, weight_decay, step, stream=None):
    """mm_gpu_clip_adamw on torch CUDA tensors (flat, tensors one after another): [norm, factor, applied]."""
    n = len(numel)
    sizes = (C.c_int64 * max(n, 1))(*numel)
    flags = (C.c_int32 * max(n, 1))(*[1 if d else 0 for d in decay])
    out = (C.c_float * 3)()
    check(load().mm_gpu_clip_adamw(n, sizes, flags, _ptr(p), _ptr(g), _ptr(m), _ptr(v), max_norm, lr, beta1, beta2,
                                   eps, weight_decay, step, out, _stream(stream)))
    return list(out)


def attention_forward(q, k, v, o, lse, *, batch, seq, n_heads, n_kv_heads, head_dim, ldq, ldk, precision=0,
                      stream=None):
    return check(load().mm_gpu_attention_forward(batch, seq, n_heads, n_kv_heads, head_dim, _ptr(q), _ptr(k), _ptr(v),
                                                 ldq, ldk, _ptr(o), _ptr(lse), precision, _stream(stream)))


def attention_backward(q, k, v, o, lse, dout, dq, dk, dv, *, batch, seq, n_heads, n_kv_heads, head_dim, ldq, ldk,
                       precision=0, stream=None):
    return check(load().mm_gpu_attention_backward(batch, seq, n_heads, n_kv_heads, head_dim, _ptr(q), _ptr(k),
                                                  _ptr(v), _ptr(o), _ptr(lse), _ptr(dout), ldq, ldk, _ptr(dq),
                                                  _ptr(dk), _ptr(dv), precision, _stream(stream)))


def attention_forward_noalloc(q, k, v, o, lse, status, *, batch, seq, n_heads, n_kv_heads, head_dim, ldq, ldk,
                              stream=None):
    """TF32 attention forward with the library's fixed score scratch (no device allocation)."""
    return check(load().mm_gpu_attention_forward_noalloc(batch, seq, n_heads, n_kv_heads, head_dim, _ptr(q), _ptr(k),
                                                         _ptr(v), ldq, ldk, _ptr(o), _ptr(lse), _ptr(status),
                                                         _stream(stream)))


def rmsnorm_forward(x, w, y, rstd, *, rows, dim, eps=1e-5, stream=None):
    return check(load().mm_gpu_rmsnorm_forward(rows, dim, _ptr(x), _ptr(w), eps, _ptr(y), _ptr(rstd),
                                               _stream(stream)))


def rmsnorm_backward(x, w, rstd, dy, dx, dw, *, rows, dim, dres=None, stream=None):
    return check(load().mm_gpu_rmsnorm_backward(rows, dim, _ptr(x), _ptr(w), _ptr(rstd), _ptr(dy), _ptr(dres),
                                                _ptr(dx), _ptr(dw), _stream(stream)))


def rope(x, cos_t, sin_t, *, rows, seq, heads, head_dim, ld, backward=False, stream=None):
    return check(load().mm_gpu_rope(rows, seq, heads, head_dim, _ptr(x), ld, _ptr(cos_t), _ptr(sin_t),
                                    int(bool(backward)), _stream(stream)))


def swiglu_forward(gate, up, act, *, n, stream=None):
    return check(load().mm_gpu_swiglu_forward(n, _ptr(gate), _ptr(up), _ptr(act), _stream(stream)))


def swiglu_backward(gate, up, dact, *, n, stream=None):
    return check(load().mm_gpu_swiglu_backward(n, _ptr(gate), _ptr(up), _ptr(dact), _stream(stream)))


def embedding_forward(ids, table, out, *, rows, vocab, dim, stream=None):
    return check(load().mm_gpu_embedding_forward(rows, _ptr(ids), vocab, dim, _ptr(table), _ptr(out),
                                                 _stream(stream)))


def embedding_backward(ids_host, dx, dtable, *, vocab, dim, stream=None):
    """ids_host: a numpy int32 array (host memory)."""
    ids = _np.ascontiguousarray(ids_host, _np.int32)
    return check(load().mm_gpu_embedding_backward(ids.size, _ip(ids), vocab, dim, _ptr(dx), _ptr(dtable),
                                                  _stream(stream)))


def cross_entropy(logits, targets, row_loss, *, rows, vocab, ld, grad_scale, mean_loss=None, stream=None):
    return check(load().mm_gpu_cross_entropy(rows, vocab, _ptr(logits), ld, _ptr(targets), grad_scale,
                                             _ptr(row_loss), _ptr(mean_loss), _stream(stream)))


class Comm:
    """mm_gpu_comm_*: one data-parallel communicator of this process's GPU."""

    def __init__(self, nccl_id: bytes, world: int, rank: int):
        idb = (C.c_uint8 * 128).from_buffer_copy(nccl_id)
        out = C.c_void_p()
        check(load().mm_gpu_comm_create(C.cast(idb, C.POINTER(C.c_uint8)), world, rank, C.byref(out)))
        self.h = out.value

    def allreduce(self, t, n=None, average=True, stream=None):
        return check(load().mm_gpu_allreduce_bucket(self.h, _ptr(t), t.numel() if n is None else n,
                                                    int(bool(average)), _stream(stream)))

    def wait(self, stream=None, timeout_ms=10_000):
        return check(load().mm_gpu_comm_wait(self.h, _stream(stream), timeout_ms))

    def close(self):
        if self.h:
            check(load().mm_gpu_comm_destroy(self.h))
            self.h = None


class Tape:
    """mm_tape_* / mm_tensor_* / mm_op_*: device tensors with a recording autograd tape on the current GPU.
    Tensors are integer handles; values and gradients cross to the host as float32 numpy arrays."""

    def __init__(self, precision: int = 0):
        self.h = load().mm_tape_create(precision)
        if self.h == 0:
            raise MidmanGpuError(-1, load().mm_gpu_last_error().decode(errors="replace"))

    def _t(self, handle):
        if handle == 0:
            raise MidmanGpuError(-1, load().mm_gpu_last_error().decode(errors="replace"))
        return handle

    def tensor(self, values=None, shape=None, requires_grad=False):
        if values is not None:
            values = _np.ascontiguousarray(values, _np.float32)
            shape = values.shape if shape is None else shape
        sh = (C.c_int64 * len(shape))(*shape)
        vp = values.ctypes.data_as(C.POINTER(C.c_float)) if values is not None else None
        return self._t(load().mm_tensor_new(self.h, sh, len(shape), vp, int(bool(requires_grad))))

    def shape(self, t):
        sh, rank = (C.c_int64 * 4)(), C.c_int32()
        check(load().mm_tensor_shape(self.h, t, sh, C.byref(rank)))
        return tuple(sh[i] for i in range(rank.value))

    def read(self, t):
        out = _np.zeros(self.shape(t), _np.float32)
        check(load().mm_tensor_read(self.h, t, out.ctypes.data_as(C.POINTER(C.c_float)), out.size))
        return out

    def grad(self, t):
        out = _np.zeros(self.shape(t), _np.float32)
        check(load().mm_tensor_grad(self.h, t, out.ctypes.data_as(C.POINTER(C.c_float)), out.size))
        return out

    def free(self, t):
        check(load().mm_tensor_free(self.h, t))

    def backward(self, loss):
        check(load().mm_tape_backward(self.h, loss))

    def matmul(self, a, b, b_transposed=False):
        return self._t(load().mm_op_matmul(self.h, a, b, int(bool(b_transposed))))

    def add(self, a, b):
        return self._t(load().mm_op_add(self.h, a, b))

    def mul(self, a, b):
        return self._t(load().mm_op_mul(self.h, a, b))

    def embedding(self, table, ids):
        ids = _np.ascontiguousarray(ids, _np.int32)
        return self._t(load().mm_op_embedding(self.h, table, _ip(ids), ids.size))

    def rms_norm(self, x, w, eps=1e-5):
        return self._t(load().mm_op_rms_norm(self.h, x, w, eps))

    def rope(self, x, seq, heads, theta=10000.0):
        return self._t(load().mm_op_rope(self.h, x, seq, heads, theta))

    def causal_attention(self, q, k, v, batch, seq, n_heads, n_kv_heads):
        return self._t(load().mm_op_causal_attention(self.h, q, k, v, batch, seq, n_heads, n_kv_heads))

    def swiglu(self, gate, up):
        return self._t(load().mm_op_swiglu(self.h, gate, up))

    def cross_entropy(self, logits, targets):
        t = _np.ascontiguousarray(targets, _np.int32)
        return self._t(load().mm_op_cross_entropy(self.h, logits, _ip(t), t.size))

    def close(self):
        if self.h:
            check(load().mm_tape_destroy(self.h))
            self.h = 0


def wait_selftest(timeout_us, stream=None):
    return check(load().mm_gpu_wait_selftest(timeout_us, _stream(stream)))


def device_status(stream=None):
    return check(load().mm_gpu_device_status(_stream(stream)))


# ---------------------------------------------------------------- midman_api.h

import json as _json

import numpy as _np


class MidmanError(RuntimeError):
    def __init__(self, status, message):
        super().__init__(f"{STATUS.get(status, status)}: {message}")
        self.status = status
        self.message = message


def text() -> str:
    L = load()
    n = L.midman_text_len()
    return C.string_at(L.midman_text_ptr(), n).decode() if n else ""


def floats() -> _np.ndarray:
    L = load()
    n = L.midman_floats_len()
    if n == 0:
        return _np.zeros(0, _np.float32)
    return _np.ctypeslib.as_array(L.midman_floats_ptr(), shape=(n,)).copy()


def error() -> str:
    L = load()
    n = L.midman_error_len()
    return C.string_at(L.midman_error_ptr(), n).decode(errors="replace") if n else ""


def api(status: int, ok=(0,)) -> int:
    if status not in ok:
        raise MidmanError(status, error())
    return status


def _dp(a):
    return a.ctypes.data_as(C.POINTER(C.c_double))


def _ip(a):
    return a.ctypes.data_as(C.POINTER(C.c_int32))


def _path_bytes(path):
    raw = str(path).encode()
    return (C.c_uint8 * len(raw)).from_buffer_copy(raw) if raw else None


def shard_inspect(path) -> dict:
    """midman_shard_inspect: {vocab_size, eos, tokens, token_width} of a checked .mmtokens file."""
    b = _path_bytes(path)
    api(load().midman_shard_inspect(b, len(b) if b is not None else 0))
    return _json.loads(text())


def shard_read(path):
    """midman_shard_read: (header dict, uint32 ids) of a checked .mmtokens file."""
    info = shard_inspect(path)
    out = _np.zeros(info["tokens"], _np.uint32)
    b = _path_bytes(path)
    api(load().midman_shard_read(b, len(b), out.ctypes.data_as(C.POINTER(C.c_uint32)), out.size))
    return _json.loads(text()), out


def shard_write(path, vocab_size: int, eos: int, tokens):
    """midman_shard_write: TokenShard::new + save."""
    t = _np.ascontiguousarray(tokens, _np.uint32)
    b = _path_bytes(path)
    api(load().midman_shard_write(b, len(b) if b is not None else 0, vocab_size, eos,
                                  t.ctypes.data_as(C.POINTER(C.c_uint32)), t.size))


def sha256(data: bytes) -> bytes:
    """midman_sha256."""
    buf = (C.c_uint8 * max(len(data), 1)).from_buffer_copy(data or b"\0")
    out = (C.c_uint8 * 32)()
    api(load().midman_sha256(buf, len(data), out))
    return bytes(out)


def shard_plan(cfg, world: int) -> dict:
    """midman_shard_plan: optimizer-sharding ranges and gradient buckets (no GPU)."""
    c = _np.ascontiguousarray(cfg, _np.float64)
    api(load().midman_shard_plan(_dp(c), world))
    return _json.loads(text())


def state_inspect(path) -> dict:
    """midman_state_inspect: the checked header of a safetensors (state) file."""
    b = _path_bytes(path)
    api(load().midman_state_inspect(b, len(b) if b is not None else 0))
    return _json.loads(text())


def config_array(vocab, d_model, n_layers, n_heads, n_kv_heads, d_ff, max_seq_len, rope_theta=10000.0,
                 norm_eps=1e-5, tie=True):
    return _np.array([vocab, d_model, n_layers, n_heads, n_kv_heads, d_ff, max_seq_len, rope_theta, norm_eps,
                      1.0 if tie else 0.0], dtype=_np.float64)


def hyper_array(max_lr=3e-4, min_lr=3e-4, warmup=0, total=1_000_000, weight_decay=0.1, clip_norm=1.0, beta1=0.9,
                beta2=0.95):
    return _np.array([max_lr, min_lr, warmup, total, weight_decay, clip_norm, beta1, beta2], dtype=_np.float64)


def describe() -> dict:
    api(load().midman_describe())
    return _json.loads(text())


def preset_config(index: int) -> _np.ndarray:
    out = _np.zeros(10, _np.float64)
    api(load().midman_preset_config(index, _dp(out)))
    return out


def config_report(cfg) -> dict:
    c = _np.ascontiguousarray(cfg, _np.float64)
    api(load().midman_config_report(_dp(c)))
    return _json.loads(text())


def rope_table(head_dim, max_seq_len, theta):
    api(load().midman_rope_table(head_dim, max_seq_len, theta))
    f = floats()
    half = head_dim // 2
    return f[: max_seq_len * half].reshape(max_seq_len, half), f[max_seq_len * half:].reshape(max_seq_len, half)


class Lab:
    """midman_lab_* (the reference's lab API) on the GPU."""

    def __init__(self, cfg, hyper, seed: int, batch: int, seq: int):
        c = _np.ascontiguousarray(cfg, _np.float64)
        h = _np.ascontiguousarray(hyper, _np.float64)
        self.h = load().midman_lab_create(_dp(c), _dp(h), seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF, batch, seq)
        if self.h == 0:
            raise MidmanError(-1, error())

    def step(self, steps: int):
        st = api(load().midman_lab_step(self.h, steps), ok=(0, 1))
        return floats().reshape(-1, 3), st, error()

    def eval(self):
        api(load().midman_lab_eval(self.h))
        return _json.loads(text())

    def stats(self):
        api(load().midman_lab_stats(self.h))
        return _json.loads(text())

    def attention(self, sequence: int):
        api(load().midman_lab_attention(self.h, sequence))
        meta = _json.loads(text())
        return floats().reshape(meta["layers"], meta["heads"], meta["seq"], meta["seq"])

    def embedding(self):
        api(load().midman_lab_embedding(self.h))
        meta = _json.loads(text())
        return floats().reshape(meta["rows"], meta["cols"])

    def close(self):
        if self.h:
            api(load().midman_lab_destroy(self.h))
            self.h = 0


def nccl_unique_id() -> bytes:
    buf = (C.c_uint8 * 128)()
    api(load().midman_nccl_unique_id(buf))
    return bytes(buf)


class Trainer:
    """midman_train_* on the current CUDA device."""

    def __init__(self, cfg, hyper, seed: int, batch: int, seq: int, precision: int = 0, world: int = 1,
                 rank: int = 0, nccl_id: bytes | None = None):
        c = _np.ascontiguousarray(cfg, _np.float64)
        h = _np.ascontiguousarray(hyper, _np.float64)
        idp = None
        if nccl_id is not None:
            self._id = (C.c_uint8 * 128).from_buffer_copy(nccl_id)
            idp = C.cast(self._id, C.POINTER(C.c_uint8))
        self.h = load().midman_train_create(_dp(c), _dp(h), seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF, batch, seq,
                                            precision, world, rank, idp)
        if self.h == 0:
            raise MidmanError(-1, error())
        self.batch, self.seq = batch, seq

    def step(self, inputs, targets):
        i = _np.ascontiguousarray(inputs, _np.int32)
        t = _np.ascontiguousarray(targets, _np.int32)
        st = api(load().midman_train_step(self.h, _ip(i), _ip(t)), ok=(0, 1))
        return floats(), st

    def stage(self, inputs, targets):
        self._si = _np.ascontiguousarray(inputs, _np.int32)
        self._st = _np.ascontiguousarray(targets, _np.int32)
        api(load().midman_train_stage(self.h, _ip(self._si), _ip(self._st)))

    def step_staged(self, steps: int = 1):
        st = api(load().midman_train_step_staged(self.h, steps), ok=(0, 1))
        return floats().reshape(-1, 3), st

    def loss_and_grads(self, inputs, targets) -> float:
        i = _np.ascontiguousarray(inputs, _np.int32)
        t = _np.ascontiguousarray(targets, _np.int32)
        api(load().midman_train_loss_and_grads(self.h, _ip(i), _ip(t)))
        return float(floats()[0])

    def read(self, which: int = 0, index: int = 0xFFFFFFFF) -> _np.ndarray:
        api(load().midman_train_read(self.h, which, index))
        return floats()

    def params(self):
        return self.read(0)

    def grads(self):
        return self.read(1)

    def load_params(self, values):
        v = _np.ascontiguousarray(values, _np.float32)
        api(load().midman_train_load(self.h, v.ctypes.data_as(C.POINTER(C.c_float)), v.size))

    def describe(self) -> dict:
        api(load().midman_train_describe(self.h))
        return _json.loads(text())

    def eval(self, inputs, targets, batch, seq) -> float:
        i = _np.ascontiguousarray(inputs, _np.int32)
        t = _np.ascontiguousarray(targets, _np.int32)
        api(load().midman_train_eval(self.h, _ip(i), _ip(t), batch, seq))
        return float(floats()[0])

    def stream(self) -> int:
        out = C.c_uint64()
        api(load().midman_train_stream(self.h, C.byref(out)))
        return out.value

    def profile(self, enable: bool):
        api(load().midman_train_profile(self.h, int(enable)))

    def run(self, batcher, steps: int):
        """midman_train_run: (records [n, 3], status, batcher place)."""
        st = api(load().midman_train_run(self.h, batcher.h, steps), ok=(0, 1))
        rec = floats().reshape(-1, 3)
        return rec, st, (_json.loads(text()) if st == 0 else None)

    def shard_optimizer(self, enable: bool = True) -> dict:
        """midman_train_shard_optimizer: ZeRO-1 on or off; returns the sharding description."""
        api(load().midman_train_shard_optimizer(self.h, 1 if enable else 0))
        return _json.loads(text())["sharding"]

    def evaluate(self, shards, max_batches: int) -> dict:
        """midman_train_evaluate: {loss, batches, tokens} over held-out shard files."""
        b = _path_bytes("\n".join(str(p) for p in shards))
        api(load().midman_train_evaluate(self.h, b, len(b) if b is not None else 0, max_batches))
        return _json.loads(text())

    def save(self, path, data_seed: int = 0, epoch: int = 0, position: int = 0):
        """Writes the run's state file (param/*, adamw.m/*, adamw.v/* and the run's metadata)."""
        b = _path_bytes(path)
        api(load().midman_train_save(self.h, b, len(b), data_seed & 0xFFFFFFFF, data_seed >> 32, epoch, position))

    def restore(self, path, data_seed: int = 0) -> dict:
        """Loads a state file into this run; returns its progress {step, epoch, position}."""
        b = _path_bytes(path)
        api(load().midman_train_restore(self.h, b, len(b), data_seed & 0xFFFFFFFF, data_seed >> 32))
        return _json.loads(text())

    def close(self):
        if self.h:
            api(load().midman_train_destroy(self.h))
            self.h = 0


class Batcher:
    """midman_batcher_*: the reference's Sequences + Batcher over token ids, synthetic ids or shard files."""

    def __init__(self, tokens=None, *, vocab=0, seq, batch, seed=0, synthetic_tokens=None, token_seed=0,
                 shards=None):
        L = load()
        s_lo, s_hi = seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF
        if shards is not None:
            b = _path_bytes("\n".join(str(p) for p in shards))
            st = L.midman_batcher_open(b, len(b) if b is not None else 0, seq, batch, s_lo, s_hi)
        elif tokens is not None:
            self._tok = _np.ascontiguousarray(tokens, _np.uint32)
            st = L.midman_batcher_create(self._tok.ctypes.data_as(C.POINTER(C.c_uint32)), self._tok.size, vocab,
                                         seq, batch, s_lo, s_hi)
        else:
            st = L.midman_batcher_synthetic(token_seed, vocab, synthetic_tokens, seq, batch, s_lo, s_hi)
        if st <= 0:
            raise MidmanError(st, error())
        self.h, self.seq, self.batch = st, seq, batch

    def next(self):
        i = _np.zeros(self.batch * self.seq, _np.int32)
        t = _np.zeros(self.batch * self.seq, _np.int32)
        api(load().midman_batcher_next(self.h, _ip(i), _ip(t)))
        meta = _json.loads(text())
        return i, t, meta["epoch"], meta["index"]

    def seek(self, epoch: int, batches_done: int) -> dict:
        api(load().midman_batcher_seek(self.h, epoch, batches_done))
        return _json.loads(text())

    def close(self):
        if self.h:
            api(load().midman_batcher_destroy(self.h))
            self.h = 0
