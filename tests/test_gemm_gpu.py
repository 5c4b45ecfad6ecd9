"""The tcgen05 TF32 GEMM against a float64 PyTorch product of the same operands.

The reference computes these products with the plain f32 loops of
crates/midman-tensor/src/kernels.rs:87-109 (gemm_nn / gemm_tn, gemm_nt through a
transposed copy, kernels.rs:66-75). TF32 keeps 10 mantissa bits per operand, so
one TF32 pass is held to relative L2 error 5e-3; the 3xTF32 split to 1e-5 (the
tolerances the training-step parity gates use for gradients).
"""
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

TF32_TOL = 5e-3
X3_TOL = 1e-5


def round4(n):
    return (n + 3) // 4 * 4


def operand(rows, cols, mn_major, gen):
    """Logical [rows x cols] (rows = M or N, cols = K) stored K- or MN-major, ld a multiple of 4."""
    if not mn_major:
        ld = round4(cols)
        store = torch.randn(rows, ld, generator=gen, device="cuda")
        return store, ld, store[:, :cols]
    ld = round4(rows)
    store = torch.randn(cols, ld, generator=gen, device="cuda")
    return store, ld, store[:, :rows].t()


def rel_l2(got, want):
    return ((got.double() - want).norm() / want.norm().clamp_min(1e-300)).item()


# From (4096, 1408, 512) on they run on CTA pairs (256 x 256 tiles): ragged M and N
# (2-D boxes for MN-major operands whose extent is not a multiple of 32), ragged K.
# On 148 SMs (74 pairs) the tiles of the last, partial wave are cut into K parts of
# at least 2,048 (summed by a second kernel): (2200, 2340, 8200) has 90 tiles, 16 of
# them in 4 parts, with ragged edges and uneven parts; (2048, 1024, 4100) 32 tiles
# in 2 parts each; (8192, 2048, 4096) 34 of 256 tiles in 2 parts. (2048, 2048, 8192)
# and (8192, 5632, 2048) are training-step shapes whose last wave stays whole (64 of
# 74 pairs busy; 38 tiles of K 2,048); (256, 512, 32768) runs on single CTAs.
SHAPES = [(128, 256, 32), (256, 512, 512), (300, 344, 200), (64, 8, 12), (1000, 1032, 1000),
          (4096, 1408, 512), (2200, 2340, 300), (2304, 4096, 64), (2200, 2340, 8200), (2048, 1024, 4100),
          (8192, 2048, 4096), (2048, 2048, 8192), (8192, 5632, 2048), (256, 512, 32768)]
MAJORS = [(False, True), (False, False), (True, True), (True, False)]


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("majors", MAJORS)
@pytest.mark.parametrize("precision", [0, 1])
def test_gemm_matches_float64(mm, shape, majors, precision):
    m, n, k = shape
    a_mn, b_mn = majors
    gen = torch.Generator(device="cuda").manual_seed(m * 7 + n * 3 + k + a_mn * 2 + b_mn)
    a_store, lda, a = operand(m, k, a_mn, gen)
    b_store, ldb, b = operand(n, k, b_mn, gen)
    ldc = round4(n)
    c = torch.full((m, ldc), float("nan"), device="cuda")
    mm.gemm(a_store, b_store, c, m=m, n=n, k=k, lda=lda, ldb=ldb, ldc=ldc,
            a_mn_major=a_mn, b_mn_major=b_mn, precision=precision)
    mm.device_status()
    want = a.double() @ b.double().t()
    got = c[:, :n]
    assert torch.isfinite(got).all()
    err = rel_l2(got, want)
    # the fp32 accumulation in TMEM adds an error that grows like sqrt(K): the
    # 3xTF32 bound is for K up to ~1,000 and is scaled beyond
    assert err < (TF32_TOL if precision == 0 else X3_TOL * max(1.0, (k / 1000) ** 0.5)), err
    if ldc > n:  # padding columns are not written
        assert torch.isnan(c[:, n:]).all()


@pytest.mark.parametrize("precision", [0, 1])
@pytest.mark.parametrize("shape", [(384, 512, 256), (2048, 1024, 4100), (2200, 2340, 8200), (8192, 2048, 2048)])
def test_gemm_adds_the_residual_in_place(mm, precision, shape):
    m, n, k = shape
    gen = torch.Generator(device="cuda").manual_seed(5)
    a = torch.randn(m, k, generator=gen, device="cuda")
    w = torch.randn(k, n, generator=gen, device="cuda")
    resid = torch.randn(m, n, generator=gen, device="cuda")
    c = resid.clone()
    mm.gemm(a, w, c, m=m, n=n, k=k, lda=k, ldb=n, ldc=n, a_mn_major=False, b_mn_major=True,
            r=c, ldr=n, precision=precision)
    mm.device_status()
    want = resid.double() + a.double() @ w.double()
    assert rel_l2(c, want) < (TF32_TOL if precision == 0 else X3_TOL * max(1.0, (k / 1000) ** 0.5))


@pytest.mark.parametrize("precision", [0, 1])
def test_gemm_empty_sizes(mm, precision):
    """M or N = 0 writes nothing; K = 0 makes C = R, or zeros without R (an empty sum)."""
    a = torch.randn(64, 32, device="cuda")
    b = torch.randn(48, 32, device="cuda")
    c = torch.full((64, 48), float("nan"), device="cuda")
    for m, n in ((0, 48), (64, 0)):
        mm.gemm(a, b, c, m=m, n=n, k=32, lda=32, ldb=32, ldc=48, a_mn_major=False, b_mn_major=False,
                precision=precision)
    mm.device_status()
    assert torch.isnan(c).all()
    r = torch.randn(64, 48, device="cuda")
    mm.gemm(a, b, c, m=64, n=48, k=0, lda=32, ldb=32, ldc=48, a_mn_major=False, b_mn_major=False, r=r, ldr=48,
            precision=precision)
    mm.device_status()
    assert torch.equal(c, r)
    mm.gemm(a, b, c, m=64, n=48, k=0, lda=32, ldb=32, ldc=48, a_mn_major=False, b_mn_major=False,
            precision=precision)
    mm.device_status()
    assert not c.any()


def test_gemm_rejects_misaligned_leading_dimensions(mm):
    a = torch.randn(16, 10, device="cuda")
    b = torch.randn(16, 12, device="cuda")
    c = torch.empty(16, 16, device="cuda")
    with pytest.raises(mm.MidmanGpuError):
        mm.gemm(a, b, c, m=16, n=16, k=10, lda=10, ldb=12, ldc=16, a_mn_major=False,
                b_mn_major=False)


# Sums of products (mm_gpu_gemm_sum): one accumulator over the terms' K steps when
# the shape runs on CTA pairs (the backward's dX = dQ Wq^T + dK Wk^T + dV Wv^T),
# ragged and zero K per term, more terms than one launch takes, narrow shapes
# that fall back to one launch per term.
SUM_CASES = [((2048, 2048), (2048, 1024, 1024)), ((2200, 2340), (300, 40, 0)), ((4096, 1408), (200, 1000)),
             ((300, 344), (64, 100)), ((2048, 1024), (4100, 2000)), ((2304, 2048), (512, 256, 128, 64))]


@pytest.mark.parametrize("case", SUM_CASES)
@pytest.mark.parametrize("majors", MAJORS)
@pytest.mark.parametrize("residual", [False, True])
def test_gemm_sum_matches_float64(mm, case, majors, residual):
    (m, n), ks = case
    a_mn, b_mn = majors
    gen = torch.Generator(device="cuda").manual_seed(m + n + sum(ks) + a_mn * 2 + b_mn)
    terms, want = [], torch.zeros(m, n, dtype=torch.float64, device="cuda")
    for k in ks:
        a_store, lda, a = operand(m, max(k, 1), a_mn, gen)
        b_store, ldb, b = operand(n, max(k, 1), b_mn, gen)
        terms.append((a_store, lda, b_store, ldb, k))
        if k:
            want += a[:, :k].double() @ b[:, :k].double().t()
    ldc = round4(n)
    r = torch.randn(m, ldc, generator=gen, device="cuda") if residual else None
    if residual:
        want += r[:, :n].double()
    c = torch.full((m, ldc), float("nan"), device="cuda")
    mm.gemm_sum(terms, c, m=m, n=n, ldc=ldc, a_mn_major=a_mn, b_mn_major=b_mn, r=r, ldr=ldc if residual else 0)
    mm.device_status()
    got = c[:, :n]
    assert torch.isfinite(got).all()
    assert rel_l2(got, want) < TF32_TOL


# the isolated Linear op fwd+bwd, X [4096 x K], W [K x N], dY [4096 x N], N(0,1) from a
# seed, checked against the reference's CPU matmul (the oracle's gemm_nn / gemm_nt / gemm_tn, which
# keep kernels.rs:87-109's per-element order): Y = X W, dX = dY W^T, dW = X^T dY.
LINEAR_SHAPES = [(512, 512), (512, 1408), (1024, 4096), (2048, 5632)]


@pytest.mark.parametrize("precision", [0, 1])
@pytest.mark.parametrize("kn", LINEAR_SHAPES)
def test_linear_config_products_match_the_reference_matmul(mm, kn, precision):
    import numpy as np
    import oracle as orc
    K, N = kn
    M = 4096
    rs = np.random.default_rng(K * 10_000 + N)
    x = rs.standard_normal((M, K), dtype=np.float32)
    w = rs.standard_normal((K, N), dtype=np.float32)
    dy = rs.standard_normal((M, N), dtype=np.float32)
    want = {"y": orc.gemm_nn(x, w), "dx": orc.gemm_nt(dy, w), "dw": orc.gemm_tn(x, dy)}
    xg, wg, dyg = (torch.from_numpy(a).cuda() for a in (x, w, dy))
    y, dx, dw = torch.empty(M, N, device="cuda"), torch.empty(M, K, device="cuda"), torch.empty(K, N, device="cuda")
    mm.gemm(xg, wg, y, m=M, n=N, k=K, lda=K, ldb=N, ldc=N, a_mn_major=False, b_mn_major=True, precision=precision)
    mm.gemm(dyg, wg, dx, m=M, n=K, k=N, lda=N, ldb=N, ldc=K, a_mn_major=False, b_mn_major=False,
            precision=precision)
    mm.gemm(xg, dyg, dw, m=K, n=N, k=M, lda=K, ldb=N, ldc=N, a_mn_major=True, b_mn_major=True, precision=precision)
    mm.device_status()
    for name, got, k in (("y", y, K), ("dx", dx, N), ("dw", dw, M)):
        ref = torch.from_numpy(want[name]).cuda().double()
        err = rel_l2(got, ref)
        # the reference's own f32 sums carry an error growing like sqrt(K) as well
        assert err < (TF32_TOL if precision == 0 else X3_TOL * max(1.0, (k / 1000) ** 0.5)), (name, err)
