"""The layer-level kernel entry points (mm_gpu_rmsnorm_*, mm_gpu_rope, mm_gpu_swiglu_*,
mm_gpu_embedding_*, mm_gpu_cross_entropy) against the oracle's restatement of the
reference's f32 layer code on the same inputs.

Gather and scatter-add are bit-exact (the scatter adds each table row's gradients in
the reference's row order); the arithmetic layers differ from the reference's f32
loops only in summation order and last-bit rounding (tree sums, fused multiply-add,
CUDA's expf), so they are held to relative L2 1e-5 (RoPE and SwiGLU, elementwise, to
1e-6). Shapes include the benchmarked ones: 8,192 tokens of d_model 1024 and 2048,
d_ff 2816 and 5632, vocabularies 32,000 and 32,768.
"""
import numpy as np
import pytest

import oracle as orc

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def rel(got, want):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    return float(np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-30))


def cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    return t.detach().cpu().numpy()


@pytest.mark.parametrize("rows,dim", [(1, 4), (37, 100), (8192, 1024), (8192, 2048), (130, 6000)])
def test_rmsnorm_forward_and_backward_match_the_reference(mm, rows, dim):
    rs = np.random.default_rng(rows * 7 + dim)
    x = rs.standard_normal((rows, dim), dtype=np.float32)
    w = rs.standard_normal(dim, dtype=np.float32)
    dy = rs.standard_normal((rows, dim), dtype=np.float32)
    res = rs.standard_normal((rows, dim), dtype=np.float32)
    want_y, want_rstd = orc.rms_norm(x, w, 1e-5)
    want_dx, want_dw = orc.rms_norm_backward(x, w, dy, 1e-5)
    xg, wg, dyg = cuda(x), cuda(w), cuda(dy)
    y, rstd = torch.empty_like(xg), torch.empty(rows, device="cuda")
    mm.rmsnorm_forward(xg, wg, y, rstd, rows=rows, dim=dim, eps=1e-5)
    dx, dw = cuda(res), torch.full((dim,), float("nan"), device="cuda")
    mm.rmsnorm_backward(xg, wg, rstd, dyg, dx, dw, rows=rows, dim=dim, dres=dx)  # dx = res + d/dx in place
    mm.device_status()
    assert rel(host(y), want_y) < 1e-5
    assert rel(host(rstd), want_rstd) < 1e-5
    assert rel(host(dx), want_dx + res) < 1e-5
    assert rel(host(dw), want_dw) < 1e-5 * max(1.0, (rows / 1000) ** 0.5)


def test_rmsnorm_refuses_unaligned_width(mm):
    x = torch.zeros(4, 6, device="cuda")
    with pytest.raises(mm.MidmanGpuError) as e:
        mm.rmsnorm_forward(x, x[0], x, x[:, 0], rows=4, dim=6)
    assert e.value.status == -3


@pytest.mark.parametrize("B,T,heads,hd", [(2, 16, 3, 8), (1, 130, 4, 64), (4, 2048, 24, 128), (8, 1024, 16, 64)])
@pytest.mark.parametrize("backward", [False, True])
def test_rope_matches_the_reference(mm, B, T, heads, hd, backward):
    rs = np.random.default_rng(B * T + heads + hd)
    x = rs.standard_normal((B, T, heads, hd), dtype=np.float32)
    cos_t, sin_t = orc.rope_table(hd, T, 10000.0)
    want = orc.rope(x.transpose(0, 2, 1, 3), cos_t, sin_t, backward).transpose(0, 2, 1, 3)
    xg = cuda(x)
    mm.rope(xg, cuda(cos_t), cuda(sin_t), rows=B * T, seq=T, heads=heads, head_dim=hd, ld=heads * hd,
            backward=backward)
    mm.device_status()
    assert rel(host(xg), want) < 1e-6


@pytest.mark.parametrize("n", [1, 7, 8192 * 2816, 8192 * 5632 + 3])
def test_swiglu_forward_and_backward_match_the_reference(mm, n):
    rs = np.random.default_rng(n % 1000)
    g = (rs.standard_normal(n, dtype=np.float32) * 3).astype(np.float32)
    u = rs.standard_normal(n, dtype=np.float32)
    d = rs.standard_normal(n, dtype=np.float32)
    want_act = orc.swiglu(g, u)
    want_dg, want_du = orc.swiglu(g, u, d)
    gg, ug = cuda(g), cuda(u)
    act = torch.empty_like(gg)
    mm.swiglu_forward(gg, ug, act, n=n)
    mm.swiglu_backward(gg, ug, cuda(d), n=n)
    mm.device_status()
    assert rel(host(act), want_act) < 1e-6
    assert rel(host(gg), want_dg) < 1e-6
    assert rel(host(ug), want_du) < 1e-6


@pytest.mark.parametrize("rows,vocab,dim", [(5, 16, 4), (8192, 32000, 2048), (2048, 4096, 128)])
def test_embedding_gather_and_scatter_add_are_bit_exact(mm, rows, vocab, dim):
    rs = np.random.default_rng(rows + vocab)
    table = rs.standard_normal((vocab, dim), dtype=np.float32)
    # many repeats of a few ids, as a batch of text has
    ids = np.concatenate([rs.integers(0, vocab, rows // 2), rs.integers(0, 8, rows - rows // 2)]).astype(np.int32)
    rs.shuffle(ids)
    dx = rs.standard_normal((rows, dim), dtype=np.float32)
    base = rs.standard_normal((vocab, dim), dtype=np.float32)
    want_out = orc.embedding(ids, table)
    want_dt = orc.embedding_backward(ids, dx, base.copy())
    out = torch.empty(rows, dim, device="cuda")
    mm.embedding_forward(cuda(ids), cuda(table), out, rows=rows, vocab=vocab, dim=dim)
    dt = cuda(base)
    mm.embedding_backward(ids, cuda(dx), dt, vocab=vocab, dim=dim)
    mm.device_status()
    assert np.array_equal(host(out).view(np.uint32), want_out.view(np.uint32))
    assert np.array_equal(host(dt).view(np.uint32), want_dt.view(np.uint32))


def test_embedding_ids_outside_the_vocabulary_are_refused(mm):
    table = torch.randn(16, 8, device="cuda")
    ids = np.array([1, 16, 3], np.int32)
    out = torch.full((3, 8), 5.0, device="cuda")
    mm.embedding_forward(cuda(ids), table, out, rows=3, vocab=16, dim=8)
    with pytest.raises(mm.MidmanGpuError, match="outside"):
        mm.device_status()
    assert (out[1] == 0).all() and torch.equal(out[0], table[1]) and torch.equal(out[2], table[3])
    dt = torch.zeros(16, 8, device="cuda")
    with pytest.raises(mm.MidmanGpuError) as e:
        mm.embedding_backward(np.array([0, -1], np.int32), torch.ones(2, 8, device="cuda"), dt, vocab=16, dim=8)
    assert e.value.status == -4
    assert (dt == 0).all()


@pytest.mark.parametrize("rows,vocab", [(3, 10), (64, 4099), (2048, 32000), (1024, 32768)])
def test_cross_entropy_matches_the_reference(mm, rows, vocab):
    rs = np.random.default_rng(rows + vocab)
    logits = (rs.standard_normal((rows, vocab), dtype=np.float32) * 2).astype(np.float32)
    targets = rs.integers(0, vocab, rows).astype(np.int32)
    want_loss, want_grad = orc.cross_entropy(logits, targets, grad=True)
    z = cuda(logits)
    row_loss = torch.empty(rows, device="cuda")
    mean = torch.zeros(1, dtype=torch.float64, device="cuda")
    mm.cross_entropy(z, cuda(targets), row_loss, rows=rows, vocab=vocab, ld=vocab, grad_scale=1.0 / rows,
                     mean_loss=mean)
    mm.device_status()
    assert abs(mean.item() - want_loss) <= 1e-6 * abs(want_loss)
    assert rel(host(z), want_grad) < 1e-5


def test_cross_entropy_target_outside_the_vocabulary(mm):
    z = torch.randn(2, 8, device="cuda")
    row_loss = torch.empty(2, device="cuda")
    mm.cross_entropy(z, cuda(np.array([3, 8], np.int32)), row_loss, rows=2, vocab=8, ld=8, grad_scale=0.5)
    with pytest.raises(mm.MidmanGpuError, match="outside"):
        mm.device_status()
    assert torch.isfinite(row_loss[0]) and torch.isnan(row_loss[1])
