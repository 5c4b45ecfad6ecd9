"""The oracle against the reference's own plain-C kernels (benches/midman-bench/c/baseline_kernels.c).

`make -C oracle ref` compiles that file, where it lies in the reference tree, into
oracle/_ref/libmidman_baseline.so. The reference keeps these C twins bit-identical
(matmul) or within 1e-6 (softmax, silu, rms_norm, adamw: they divide where the Rust
multiplies by an inverse) of its Rust kernels, so the same bars apply to the oracle.
"""
import ctypes as C
from pathlib import Path

import numpy as np
import pytest

import oracle as orc

REF = Path(__file__).resolve().parent.parent / "oracle" / "_ref" / "libmidman_baseline.so"
pytestmark = pytest.mark.skipif(not REF.exists(), reason="reference C baselines not built (make -C oracle ref)")

F = C.POINTER(C.c_float)


@pytest.fixture(scope="module")
def ref():
    lib = C.CDLL(str(REF))
    lib.mmb_matmul_ikj.argtypes = [F, F, F, C.c_size_t]
    lib.mmb_softmax_rows.argtypes = [F, F, C.c_size_t, C.c_size_t]
    lib.mmb_silu.argtypes = [F, F, C.c_size_t]
    lib.mmb_rms_norm.argtypes = [F, F, F, C.c_size_t, C.c_size_t, C.c_float]
    lib.mmb_adamw_update.argtypes = [F, F, F, F, C.c_size_t, C.c_int, C.c_float, C.c_float, C.c_float, C.c_float,
                                     C.c_float]
    return lib


def p(a):
    return a.ctypes.data_as(F)


def test_matmul_bit_identical(ref):
    rng = np.random.default_rng(1)
    for n in (1, 7, 33, 64):
        a = rng.standard_normal((n, n)).astype(np.float32)
        b = rng.standard_normal((n, n)).astype(np.float32)
        c = np.zeros((n, n), np.float32)
        ref.mmb_matmul_ikj(p(a), p(b), p(c), n)
        assert np.array_equal(orc.gemm_nn(a, b).view(np.uint32), c.view(np.uint32))


def test_softmax_matches(ref):
    x = np.random.default_rng(2).standard_normal((16, 300)).astype(np.float32) * 4
    y = np.zeros_like(x)
    ref.mmb_softmax_rows(p(x), p(y), 16, 300)
    np.testing.assert_allclose(orc.softmax_rows(x), y, rtol=1e-6, atol=1e-9)


def test_cross_entropy_gradient_is_softmax_minus_onehot(ref):
    x = np.random.default_rng(3).standard_normal((8, 50)).astype(np.float32)
    t = np.arange(8, dtype=np.int32) * 5
    y = np.zeros_like(x)
    ref.mmb_softmax_rows(p(x), p(y), 8, 50)
    _, g = orc.cross_entropy(x, t, grad=True)
    y[np.arange(8), t] -= 1.0
    np.testing.assert_allclose(g, y / 8, rtol=1e-5, atol=1e-8)


def test_rms_norm_forward_matches(ref):
    # the oracle's model path through rms_norm is checked through a one-layer model's logits
    # elsewhere; here the primitive chain itself, via a d_model x 1-row model is overkill, so
    # compare the formula: the C twin against numpy's float32 evaluation of the same chain.
    x = np.random.default_rng(4).standard_normal((10, 64)).astype(np.float32)
    w = np.random.default_rng(5).standard_normal(64).astype(np.float32)
    out = np.zeros_like(x)
    ref.mmb_rms_norm(p(x), p(w), p(out), 10, 64, np.float32(1e-5))
    ms = (x * x).sum(-1, dtype=np.float32) * np.float32(1 / 64)
    inv = np.power(ms + np.float32(1e-5), np.float32(-0.5))
    np.testing.assert_allclose((x * inv[:, None]) * w, out, rtol=2e-6, atol=1e-7)


def test_adamw_matches(ref):
    rng = np.random.default_rng(6)
    n = 1000
    w0 = rng.standard_normal(n).astype(np.float32)
    wa, wb = w0.copy(), w0.copy()
    ma, va, mb, vb = (np.zeros(n, np.float32) for _ in range(4))
    for step in range(1, 6):
        g = rng.standard_normal(n).astype(np.float32)
        ref.mmb_adamw_update(p(wa), p(g), p(ma), p(va), n, step, 1e-3, 0.9, 0.95, 1e-8, 0.1)
        orc.adamw_update(wb, g, mb, vb, True, step, 1e-3, 0.9, 0.95, 1e-8, 0.1)
    np.testing.assert_allclose(wb, wa, rtol=1e-6, atol=1e-8)
