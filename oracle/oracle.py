"""ctypes binding of the CPU oracle (oracle/_build/liboracle.so) -- TEST INFRASTRUCTURE.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this
module, as the checker or the timed CPU baseline. See oracle.h for what the
oracle restates and where in the reference each part comes from.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "_build" / "liboracle.so"
_lib = None


def build() -> Path:
    r = subprocess.run(["make", "-C", str(HERE), "-j8", "all"], capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{r.stdout}\n{r.stderr}")
    return LIB


def lib() -> C.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not LIB.exists():
        build()
    L = C.CDLL(str(LIB))
    vp, u64, f32, f64, i32, sz = C.c_void_p, C.c_uint64, C.c_float, C.c_double, C.c_int, C.c_size_t
    P = C.POINTER

    def sig(name, res, *args):
        f = getattr(L, name)
        f.restype = res
        f.argtypes = list(args)

    sig("or_set_threads", None, i32)
    sig("or_rng_new", vp, u64)
    sig("or_rng_free", None, vp)
    sig("or_rng_next_u64", u64, vp)
    sig("or_rng_next_f32", f32, vp)
    sig("or_rng_next_f64", f64, vp)
    sig("or_rng_uniform", f32, vp, f32, f32)
    sig("or_rng_normal", f32, vp)
    sig("or_rng_below", u64, vp, u64)
    sig("or_rng_shuffle", None, vp, P(u64), sz)
    sig("or_rng_fork", vp, vp, u64)
    sig("or_param_breakdown", i32, P(f64), P(u64), C.c_char_p, sz)
    sig("or_rope_table", i32, i32, i32, f32, P(f32), P(f32))
    sig("or_model_new", vp, P(f64), vp, f32)
    sig("or_model_free", None, vp)
    sig("or_model_num_params", sz, vp)
    sig("or_model_num_tensors", i32, vp)
    sig("or_model_param_info", i32, vp, i32, C.c_char_p, sz, P(i32), P(C.c_int64), P(u64), P(u64))
    sig("or_model_get_params", None, vp, P(f32))
    sig("or_model_set_params", None, vp, P(f32))
    sig("or_model_loss", i32, vp, P(C.c_int32), P(C.c_int32), i32, i32, P(f32), P(f32))
    sig("or_model_logits", i32, vp, P(C.c_int32), i32, i32, P(f32))
    sig("or_model_attention", i32, vp, P(C.c_int32), i32, i32, P(f32))
    sig("or_clip_global_norm", f32, P(f32), sz, f32, P(i32))
    sig("or_schedule_lr", f32, f32, f32, u64, u64, u64)
    sig("or_adamw_new", vp, vp, f32, f32, f32, f32)
    sig("or_adamw_free", None, vp)
    sig("or_adamw_step", i32, vp, vp, P(f32), f32)
    sig("or_adamw_steps", u64, vp)
    sig("or_adamw_moments", None, vp, P(f32), P(f32))
    sig("or_adamw_restore", i32, vp, u64, P(f32), P(f32))
    sig("or_train_update", i32, vp, vp, P(C.c_int32), P(C.c_int32), i32, i32, f32, f32, P(f32))
    sig("or_batcher_new", vp, P(C.c_uint32), sz, i32, i32, u64)
    sig("or_batcher_new_shards", vp, P(C.c_uint32), P(sz), sz, i32, i32, u64)
    sig("or_batcher_free", None, vp)
    sig("or_batcher_num_sequences", sz, vp)
    sig("or_batcher_next", None, vp, P(C.c_int32), P(C.c_int32), P(u64), P(u64))
    sig("or_gemm_nn", None, P(f32), P(f32), P(f32), sz, sz, sz)
    sig("or_gemm_nt", None, P(f32), P(f32), P(f32), sz, sz, sz)
    sig("or_gemm_tn", None, P(f32), P(f32), P(f32), sz, sz, sz)
    sig("or_softmax_rows", None, P(f32), P(f32), sz, sz)
    sig("or_cross_entropy", f32, P(f32), P(C.c_int32), sz, sz, P(f32))
    sig("or_causal_attention", i32, P(f64), P(f32), P(f32), P(f32), i32, i32, P(f32), P(f32))
    sig("or_adamw_update", i32, P(f32), P(f32), P(f32), P(f32), sz, i32, u64, f32, f32, f32, f32, f32)
    sig("or_rms_norm", None, P(f32), P(f32), sz, sz, f32, P(f32), P(f32))
    sig("or_rms_norm_bwd", None, P(f32), P(f32), P(f32), sz, sz, f32, P(f32), P(f32))
    sig("or_rope", None, P(f32), sz, sz, sz, P(f32), P(f32), i32)
    sig("or_swiglu", None, P(f32), P(f32), sz, P(f32), P(f32), P(f32), P(f32))
    sig("or_embedding", None, P(C.c_int32), sz, P(f32), sz, P(f32), P(f32), P(f32))
    _lib = L
    return L


def _p(a: np.ndarray, ct):
    return a.ctypes.data_as(C.POINTER(ct))


def set_threads(n: int) -> None:
    lib().or_set_threads(int(n))


class Rng:
    """crates/midman-foundation/src/rng.rs Rng."""

    def __init__(self, seed: int = 0, _handle=None):
        self.h = _handle if _handle is not None else lib().or_rng_new(C.c_uint64(seed & (2**64 - 1)))

    def __del__(self):
        if getattr(self, "h", None):
            lib().or_rng_free(self.h)
            self.h = None

    def next_u64(self):
        return lib().or_rng_next_u64(self.h)

    def next_f32(self):
        return lib().or_rng_next_f32(self.h)

    def next_f64(self):
        return lib().or_rng_next_f64(self.h)

    def uniform(self, lo, hi):
        return lib().or_rng_uniform(self.h, lo, hi)

    def normal(self):
        return lib().or_rng_normal(self.h)

    def below(self, n):
        return lib().or_rng_below(self.h, n)

    def shuffle(self, items):
        a = np.ascontiguousarray(items, dtype=np.uint64)
        lib().or_rng_shuffle(self.h, _p(a, C.c_uint64), a.size)
        return a

    def fork(self, stream):
        return Rng(_handle=lib().or_rng_fork(self.h, stream))


def config_array(vocab, d_model, n_layers, n_heads, n_kv_heads, d_ff, max_seq_len, rope_theta=10000.0,
                 norm_eps=1e-5, tie=True):
    return np.array([vocab, d_model, n_layers, n_heads, n_kv_heads, d_ff, max_seq_len, rope_theta, norm_eps,
                     1.0 if tie else 0.0], dtype=np.float64)


PRESETS = {  # crates/midman-model-config/src/presets.rs:61-83
    "smoke": (256, 64, 2, 4, 4, 176, 128),
    "tiny": (4096, 128, 4, 4, 4, 344, 256),
    "small": (32000, 384, 6, 6, 6, 1024, 512),
    "base": (32000, 768, 12, 12, 12, 2048, 1024),
    "medium": (32000, 1024, 24, 16, 8, 2816, 2048),
    "large": (32000, 2048, 20, 16, 8, 5632, 2048),
}


def preset(name: str, vocab: int | None = None) -> np.ndarray:
    v, d, l, h, kv, ff, t = PRESETS[name]
    return config_array(vocab or v, d, l, h, kv, ff, t)


def param_breakdown(cfg: np.ndarray):
    out = np.zeros(6, dtype=np.uint64)
    msg = C.create_string_buffer(64)
    rc = lib().or_param_breakdown(_p(np.ascontiguousarray(cfg, np.float64), C.c_double), _p(out, C.c_uint64),
                                  msg, 64)
    if rc:
        raise ValueError(msg.value.decode())
    keys = ["embedding", "attention", "mlp", "norms", "lm_head", "total"]
    return {k: int(v) for k, v in zip(keys, out)}


def rope_table(head_dim, max_seq_len, theta):
    half = head_dim // 2
    c = np.zeros(max_seq_len * half, np.float32)
    s = np.zeros(max_seq_len * half, np.float32)
    if lib().or_rope_table(head_dim, max_seq_len, theta, _p(c, C.c_float), _p(s, C.c_float)):
        raise ValueError("bad rope arguments")
    return c.reshape(max_seq_len, half), s.reshape(max_seq_len, half)


class Model:
    """MidManModel built from Rng(seed) (or a given Rng), flat parameters in reference order."""

    def __init__(self, cfg: np.ndarray, seed: int | None = 0, rng: Rng | None = None, init_std: float = 0.02):
        self.cfg = np.ascontiguousarray(cfg, np.float64)
        self.rng = rng if rng is not None else Rng(seed)
        self.h = lib().or_model_new(_p(self.cfg, C.c_double), self.rng.h, init_std)
        if not self.h:
            raise ValueError("invalid model config")
        self.n = lib().or_model_num_params(self.h)
        self.vocab = int(self.cfg[0])

    def __del__(self):
        if getattr(self, "h", None):
            lib().or_model_free(self.h)
            self.h = None

    def tensors(self):
        out = []
        name = C.create_string_buffer(128)
        rank = C.c_int()
        shape = (C.c_int64 * 4)()
        off, num = C.c_uint64(), C.c_uint64()
        for i in range(lib().or_model_num_tensors(self.h)):
            lib().or_model_param_info(self.h, i, name, 128, C.byref(rank), shape, C.byref(off), C.byref(num))
            out.append((name.value.decode(), tuple(shape[k] for k in range(rank.value)), off.value, num.value))
        return out

    @property
    def params(self) -> np.ndarray:
        a = np.zeros(self.n, np.float32)
        lib().or_model_get_params(self.h, _p(a, C.c_float))
        return a

    @params.setter
    def params(self, a: np.ndarray):
        a = np.ascontiguousarray(a, np.float32)
        assert a.size == self.n
        lib().or_model_set_params(self.h, _p(a, C.c_float))

    def loss(self, inputs, targets, batch, seq, grads: bool = False, out=None):
        """(loss, gradients) or loss; `out` (float32, n values) receives the gradients when given."""
        i = np.ascontiguousarray(inputs, np.int32)
        t = np.ascontiguousarray(targets, np.int32)
        loss = np.zeros(1, np.float32)
        g = None
        if grads:
            g = out if out is not None else np.zeros(self.n, np.float32)
            assert g.dtype == np.float32 and g.size == self.n and g.flags.c_contiguous
        rc = lib().or_model_loss(self.h, _p(i, C.c_int32), _p(t, C.c_int32), batch, seq, _p(loss, C.c_float),
                                 _p(g, C.c_float) if grads else None)
        if rc:
            raise ValueError(f"or_model_loss failed: {rc}")
        return (float(loss[0]), g) if grads else float(loss[0])

    def logits(self, inputs, batch, seq):
        i = np.ascontiguousarray(inputs, np.int32)
        out = np.zeros(batch * seq * self.vocab, np.float32)
        if lib().or_model_logits(self.h, _p(i, C.c_int32), batch, seq, _p(out, C.c_float)):
            raise ValueError("or_model_logits failed")
        return out.reshape(batch, seq, self.vocab)

    def attention(self, inputs, batch, seq):
        layers, heads = int(self.cfg[2]), int(self.cfg[3])
        i = np.ascontiguousarray(inputs, np.int32)
        out = np.zeros(layers * batch * heads * seq * seq, np.float32)
        if lib().or_model_attention(self.h, _p(i, C.c_int32), batch, seq, _p(out, C.c_float)):
            raise ValueError("or_model_attention failed")
        return out.reshape(layers, batch, heads, seq, seq)


def _f32(a):
    return np.ascontiguousarray(a, np.float32)


def gemm_nn(a, b):
    """C = A B for A [m,k], B [k,n] (kernels.rs:90-98)."""
    a, b = _f32(a), _f32(b)
    (m, k), n = a.shape, b.shape[1]
    c = np.zeros((m, n), np.float32)
    lib().or_gemm_nn(_p(a, C.c_float), _p(b, C.c_float), _p(c, C.c_float), m, k, n)
    return c


def gemm_nt(a, b):
    """C = A B^T for A [m,k], B [n,k] (kernels.rs:66-75)."""
    a, b = _f32(a), _f32(b)
    (m, k), n = a.shape, b.shape[0]
    c = np.zeros((m, n), np.float32)
    lib().or_gemm_nt(_p(a, C.c_float), _p(b, C.c_float), _p(c, C.c_float), m, k, n)
    return c


def gemm_tn(a, b):
    """C = A^T B for A [k,m], B [k,n] (kernels.rs:101-109)."""
    a, b = _f32(a), _f32(b)
    (k, m), n = a.shape, b.shape[1]
    c = np.zeros((m, n), np.float32)
    lib().or_gemm_tn(_p(a, C.c_float), _p(b, C.c_float), _p(c, C.c_float), k, m, n)
    return c


def softmax_rows(x):
    x = _f32(x)
    y = np.zeros_like(x)
    lib().or_softmax_rows(_p(x, C.c_float), _p(y, C.c_float), x.shape[0], x.shape[1])
    return y


def cross_entropy(logits, targets, grad=False):
    x = _f32(logits)
    t = np.ascontiguousarray(targets, np.int32)
    g = np.zeros_like(x) if grad else None
    loss = lib().or_cross_entropy(_p(x, C.c_float), _p(t, C.c_int32), x.shape[0], x.shape[1],
                                  _p(g, C.c_float) if grad else None)
    return (loss, g) if grad else loss


def causal_attention(q, k, v, n_heads, n_kv_heads):
    """q [B,H,T,hd], k/v [B,Hkv,T,hd] -> (out [B,H,T,hd], probs [B,H,T,T])."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    B, H, T, hd = q.shape
    cfg = config_array(16, H * hd, 1, n_heads, n_kv_heads, 4, T)
    out = np.zeros_like(q)
    probs = np.zeros((B, H, T, T), np.float32)
    rc = lib().or_causal_attention(_p(cfg, C.c_double), _p(q, C.c_float), _p(k, C.c_float), _p(v, C.c_float), B, T,
                                   _p(out, C.c_float), _p(probs, C.c_float))
    if rc:
        raise ValueError("bad attention config")
    return out, probs


def rms_norm(x, w, eps=1e-5):
    """norm.rs:21-39 on rows of x [rows, d]: (y, rstd per row)."""
    x, w = _f32(x), _f32(w)
    rows, d = x.shape
    y = np.zeros_like(x)
    rstd = np.zeros(rows, np.float32)
    lib().or_rms_norm(_p(x, C.c_float), _p(w, C.c_float), rows, d, eps, _p(y, C.c_float), _p(rstd, C.c_float))
    return y, rstd


def rms_norm_backward(x, w, dy, eps=1e-5):
    """The reference autograd of rms_norm: (dx, dw)."""
    x, w, dy = _f32(x), _f32(w), _f32(dy)
    rows, d = x.shape
    dx = np.zeros_like(x)
    dw = np.zeros(d, np.float32)
    lib().or_rms_norm_bwd(_p(x, C.c_float), _p(w, C.c_float), _p(dy, C.c_float), rows, d, eps, _p(dx, C.c_float),
                          _p(dw, C.c_float))
    return dx, dw


def rope(x, cos_t, sin_t, backward=False):
    """apply_rope (rope.rs:20-33) or its gradient on x [B, heads, T, hd]; returns a new array."""
    y = np.array(x, np.float32, copy=True, order="C")
    B, Hh, T, hd = y.shape
    c, s = _f32(cos_t), _f32(sin_t)
    lib().or_rope(_p(y, C.c_float), B * Hh, T, hd, _p(c, C.c_float), _p(s, C.c_float), int(bool(backward)))
    return y


def swiglu(g, u, dact=None):
    """mlp.rs:20-24: act = silu(g) * u, or with dact the gradients (dg, du)."""
    g, u = _f32(g), _f32(u)
    n = g.size
    if dact is None:
        act = np.zeros_like(g)
        lib().or_swiglu(_p(g, C.c_float), _p(u, C.c_float), n, _p(act, C.c_float), None, None, None)
        return act
    dact = _f32(dact)
    dg, du = np.zeros_like(g), np.zeros_like(u)
    lib().or_swiglu(_p(g, C.c_float), _p(u, C.c_float), n, None, _p(dact, C.c_float), _p(dg, C.c_float),
                    _p(du, C.c_float))
    return dg, du


def embedding(ids, table):
    """ops_shape.rs:230-255: table[ids]."""
    ids = np.ascontiguousarray(ids, np.int32)
    table = _f32(table)
    out = np.zeros((ids.size, table.shape[1]), np.float32)
    lib().or_embedding(_p(ids, C.c_int32), ids.size, _p(table, C.c_float), table.shape[1], _p(out, C.c_float), None,
                       None)
    return out


def embedding_backward(ids, dx, dtable):
    """ops_shape.rs:262-272: dtable[ids[r]] += dx[r] in row order, in place on dtable."""
    ids = np.ascontiguousarray(ids, np.int32)
    dx = _f32(dx)
    assert dtable.dtype == np.float32 and dtable.flags.c_contiguous
    lib().or_embedding(_p(ids, C.c_int32), ids.size, None, dtable.shape[1], None, _p(dx, C.c_float),
                       _p(dtable, C.c_float))
    return dtable


def adamw_update(x, g, m, v, decay, step, lr, beta1, beta2, eps, wd):
    """In place on float32 arrays x, m, v."""
    g = _f32(g)
    lib().or_adamw_update(_p(x, C.c_float), _p(g, C.c_float), _p(m, C.c_float), _p(v, C.c_float), x.size,
                          int(decay), step, lr, beta1, beta2, eps, wd)


def clip_global_norm(grads: np.ndarray, max_norm: float):
    ok = C.c_int()
    norm = lib().or_clip_global_norm(_p(grads, C.c_float), grads.size, max_norm, C.byref(ok))
    return norm, bool(ok.value)


def schedule_lr(max_lr, min_lr, warmup, total, step):
    return lib().or_schedule_lr(max_lr, min_lr, warmup, total, step)


class AdamW:
    def __init__(self, model: Model, beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.1):
        self.model = model
        self.h = lib().or_adamw_new(model.h, beta1, beta2, eps, weight_decay)

    def __del__(self):
        if getattr(self, "h", None):
            lib().or_adamw_free(self.h)
            self.h = None

    def step(self, grads: np.ndarray, lr: float) -> bool:
        g = np.ascontiguousarray(grads, np.float32)
        return lib().or_adamw_step(self.h, self.model.h, _p(g, C.c_float), lr) == 0

    def moments(self):
        m = np.zeros(self.model.n, np.float32)
        v = np.zeros(self.model.n, np.float32)
        lib().or_adamw_moments(self.h, _p(m, C.c_float), _p(v, C.c_float))
        return m, v

    @property
    def steps(self) -> int:
        return int(lib().or_adamw_steps(self.h))

    def restore(self, steps: int, m: np.ndarray, v: np.ndarray):
        """AdamW::restore (adamw.rs:95-130) of the flat moments."""
        m = np.ascontiguousarray(m, np.float32)
        v = np.ascontiguousarray(v, np.float32)
        assert m.size == self.model.n and v.size == self.model.n
        if lib().or_adamw_restore(self.h, steps, _p(m, C.c_float), _p(v, C.c_float)) != 0:
            raise ValueError("adamw: moments are not finite or a second moment is negative")


def train_update(model: Model, opt: AdamW, inputs, targets, batch, seq, clip_norm, lr):
    """One Trainer::update: returns (loss, grad_norm, ok)."""
    i = np.ascontiguousarray(inputs, np.int32)
    t = np.ascontiguousarray(targets, np.int32)
    out = np.zeros(2, np.float32)
    rc = lib().or_train_update(model.h, opt.h, _p(i, C.c_int32), _p(t, C.c_int32), batch, seq, clip_norm, lr,
                               _p(out, C.c_float))
    return float(out[0]), float(out[1]), rc == 0


class Batcher:
    def __init__(self, tokens, seq, batch, seed, shard_lengths=None):
        """tokens: one shard, or the shards one after another with their lengths in shard_lengths."""
        self.tok = np.ascontiguousarray(tokens, np.uint32)
        self.seq, self.batch = seq, batch
        if shard_lengths is None:
            self.h = lib().or_batcher_new(_p(self.tok, C.c_uint32), self.tok.size, seq, batch, seed)
        else:
            lens = (C.c_size_t * len(shard_lengths))(*shard_lengths)
            self.h = lib().or_batcher_new_shards(_p(self.tok, C.c_uint32), lens, len(shard_lengths), seq, batch,
                                                 seed)
        if not self.h:
            raise ValueError("fewer sequences than one batch")

    def __del__(self):
        if getattr(self, "h", None):
            lib().or_batcher_free(self.h)
            self.h = None

    def __len__(self):
        return lib().or_batcher_num_sequences(self.h)

    def next(self):
        i = np.zeros(self.batch * self.seq, np.int32)
        t = np.zeros(self.batch * self.seq, np.int32)
        e, x = C.c_uint64(), C.c_uint64()
        lib().or_batcher_next(self.h, _p(i, C.c_int32), _p(t, C.c_int32), C.byref(e), C.byref(x))
        return i, t, e.value, x.value


def lab_task(cfg: np.ndarray, seed: int, batch: int, seq: int, init_std: float = 0.02):
    """Lab::new's model and task (crates/midman-api/src/lab.rs:194-204): init, then ids."""
    rng = Rng(seed)
    model = Model(cfg, rng=rng, init_std=init_std)
    vocab = int(cfg[0])
    inputs, targets = [], []
    for _ in range(batch):
        toks = [rng.below(vocab) for _ in range(seq + 1)]
        inputs += toks[:seq]
        targets += toks[1:]
    return model, np.array(inputs, np.int32), np.array(targets, np.int32)
