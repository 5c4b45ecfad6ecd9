"""mm_gpu_clip_adamw, the kernel-level clip + AdamW entry point, against the oracle.

The oracle restates clip.rs:29-59 (f64 norm, scale by max/(norm+1e-6) above max)
and adamw.rs:141-217 (decoupled decay for rank >= 2 tensors, f64 bias
corrections); the device version sums the norm over a fixed grid instead of in
order, so the norm agrees to f32 rounding and the updated values to a few ulps.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def test_clip_adamw_matches_the_oracle(mm):
    import oracle as orc
    sizes = [8, 12, 4, 1000, 30001]
    decay = [False, True, False, True, True]
    r = np.random.default_rng(3)
    p = r.standard_normal(sum(sizes)).astype(np.float32)
    m = np.zeros_like(p)
    v = np.zeros_like(p)
    dp, dm, dv = (torch.from_numpy(a.copy()).cuda() for a in (p, m, v))
    hyper = dict(lr=0.01, beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.1)
    for step, scale in ((1, 0.05), (2, 0.0001), (3, 0.02)):  # the first and last steps clip
        g = (r.standard_normal(p.size) * scale).astype(np.float32)
        norm, factor, applied = mm.clip_adamw(dp, torch.from_numpy(g).cuda(), dm, dv, sizes, decay, max_norm=1.0,
                                              step=step, **hyper)
        gc = g.copy()
        want_norm, ok = orc.clip_global_norm(gc, 1.0)
        assert ok and applied == 1.0
        assert abs(norm - want_norm) <= 1e-6 * want_norm
        assert (factor < 1.0) == (want_norm > 1.0)
        off = 0
        for n, d in zip(sizes, decay):
            sl = slice(off, off + n)
            x, mm_, vv = p[sl].copy(), m[sl].copy(), v[sl].copy()
            orc.adamw_update(x, gc[sl], mm_, vv, d, step, hyper["lr"], hyper["beta1"], hyper["beta2"], hyper["eps"],
                             hyper["weight_decay"])
            p[sl], m[sl], v[sl] = x, mm_, vv
            off += n
        for got, want in ((dp, p), (dm, m), (dv, v)):
            g_np = got.cpu().numpy()
            assert np.max(np.abs(g_np - want)) <= 1e-6 * (1.0 + np.max(np.abs(want)))
    # a non-finite gradient changes nothing (clip.rs:49-51, adamw.rs:176-181)
    before = [t.clone() for t in (dp, dm, dv)]
    g = np.zeros(p.size, np.float32)
    g[5] = np.inf
    norm, factor, applied = mm.clip_adamw(dp, torch.from_numpy(g).cuda(), dm, dv, sizes, decay, max_norm=1.0,
                                          step=4, **hyper)
    assert applied == 0.0 and not np.isfinite(norm)
    for t, b in zip((dp, dm, dv), before):
        assert torch.equal(t, b)
    with pytest.raises(mm.MidmanGpuError):  # a tensor that breaks 16-byte alignment for the next one
        mm.clip_adamw(dp, torch.from_numpy(g).cuda(), dm, dv, [5, 3], [True, True], max_norm=1.0, step=1, **hyper)
