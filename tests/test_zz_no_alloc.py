"""mm_gpu_attention_forward_noalloc against mm_gpu_attention_forward (TF32).

The allocation-free entry point runs the same tensor-core attention forward with
its score scratch in a fixed array inside the library. Two calls in a row (the
second on a smaller problem, so the shared array still holds the first call's
scores) must each match the allocating entry point within the TF32 attention
tolerance of test_attention_gpu.py; sizes past the array's limit are refused.
"""
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

TOL = 5e-3  # relative L2, as for MM_GPU_TF32 attention elsewhere in the tests


def rel(a, b):
    return ((a.double() - b.double()).norm() / b.double().norm()).item()


def inputs(B, T, H, Hkv, hd, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn(B, T, H, hd, device="cuda", generator=g)
    k = torch.randn(B, T, Hkv, hd, device="cuda", generator=g)
    v = torch.randn(B, T, Hkv, hd, device="cuda", generator=g)
    return q, k, v


def test_noalloc_matches_allocating_entry_point(mm):
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    # head_dim 32, 64 and 128 (the O = PV product's two tile widths); the last case is
    # smaller than the first, so the shared array still holds older scores
    for n, (B, T, H, Hkv, hd) in enumerate([(1, 512, 8, 2, 128), (2, 300, 4, 1, 32), (3, 77, 6, 3, 64)]):
        q, k, v = inputs(B, T, H, Hkv, hd, seed=17 + n)
        kw = dict(batch=B, seq=T, n_heads=H, n_kv_heads=Hkv, head_dim=hd, ldq=H * hd, ldk=Hkv * hd)
        o_ref, lse_ref = torch.empty(B, T, H, hd, device="cuda"), torch.empty(B, H, T, device="cuda")
        mm.attention_forward(q, k, v, o_ref, lse_ref, precision=0, **kw)
        o = torch.full_like(o_ref, float("nan"))
        lse = torch.full_like(lse_ref, float("nan"))
        mm.attention_forward_noalloc(q, k, v, o, lse, status, **kw)
        torch.cuda.synchronize()
        mm.device_status()
        assert status.item() == 0
        assert torch.isfinite(o).all() and torch.isfinite(lse).all()
        assert rel(o, o_ref) < TOL
        assert (lse - lse_ref).abs().max().item() < 1e-2


def test_noalloc_refuses_sizes_past_its_scratch(mm):
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    B, T, H, Hkv, hd = 1, 2048, 4, 2, 128  # 4 * 2048 * 2048 floats > 4194304
    q, k, v = inputs(B, T, H, Hkv, hd, seed=3)
    o, lse = torch.empty(B, T, H, hd, device="cuda"), torch.empty(B, H, T, device="cuda")
    kw = dict(batch=B, seq=T, n_heads=H, n_kv_heads=Hkv, head_dim=hd, ldq=H * hd, ldk=Hkv * hd)
    with pytest.raises(mm.MidmanGpuError, match="exceeds the fixed score scratch"):
        mm.attention_forward_noalloc(q, k, v, o, lse, status, **kw)
    kw.update(head_dim=16, ldq=H * 16, ldk=Hkv * 16)
    q, k, v = inputs(1, 64, H, Hkv, 16, seed=4)
    with pytest.raises(mm.MidmanGpuError, match="head_dim must be 32, 64 or 128"):
        mm.attention_forward_noalloc(q, k, v, o, lse, status, **dict(kw, seq=64))
    # row strides that TMA cannot address, and a misaligned output: refused before anything runs
    q, k, v = inputs(1, 64, 2, 2, 64, seed=5)
    o, lse = torch.full((1, 64, 2, 64), 7.0, device="cuda"), torch.full((1, 2, 64), 7.0, device="cuda")
    kw = dict(batch=1, seq=64, n_heads=2, n_kv_heads=2, head_dim=64, ldq=128, ldk=128)
    with pytest.raises(mm.MidmanGpuError, match="multiples of 4"):
        mm.attention_forward_noalloc(q, k, v, o, lse, status, **dict(kw, ldq=130))
    o_flat = torch.full((64 * 128 + 1,), 7.0, device="cuda")
    with pytest.raises(mm.MidmanGpuError, match="16-byte aligned"):
        mm.attention_forward_noalloc(q, k, v, o_flat[1:], lse, status, **kw)
    torch.cuda.synchronize()
    assert (lse == 7.0).all() and (o_flat == 7.0).all()


FRESH = r"""
import sys, torch
sys.path.insert(0, sys.argv[1])
import midman_b200 as mm
torch.cuda.init()
B, T, H, Hkv, hd = 2, 256, 4, 2, 64
g = torch.Generator(device="cuda").manual_seed(1)
q = torch.randn(B, T, H, hd, device="cuda", generator=g)
k = torch.randn(B, T, Hkv, hd, device="cuda", generator=g)
v = torch.randn(B, T, Hkv, hd, device="cuda", generator=g)
o, lse = torch.empty_like(q), torch.empty(B, H, T, device="cuda")
status = torch.zeros(1, dtype=torch.int32, device="cuda")
kw = dict(batch=B, seq=T, n_heads=H, n_kv_heads=Hkv, head_dim=hd, ldq=H * hd, ldk=Hkv * hd)
mm.attention_forward_noalloc(q, k, v, o, lse, status, **kw)  # first call: loads the kernels
torch.cuda.synchronize()
free0 = torch.cuda.mem_get_info()[0]
for _ in range(3):
    mm.attention_forward_noalloc(q, k, v, o, lse, status, **kw)
torch.cuda.synchronize()
free1 = torch.cuda.mem_get_info()[0]
assert status.item() == 0 and torch.isfinite(o).all()
print("FREE", free0, free1)
"""


def test_noalloc_in_a_fresh_process_takes_no_device_memory(mm, tmp_path):
    """Called first thing in a new process, repeated calls leave the device's free memory unchanged."""
    import subprocess
    import sys
    from pathlib import Path
    script = tmp_path / "fresh.py"
    script.write_text(FRESH)
    pkg = Path(mm.__file__).resolve().parent
    r = subprocess.run([sys.executable, str(script), str(pkg)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    free0, free1 = (int(x) for x in r.stdout.split("FREE")[1].split())
    assert free0 == free1, (free0, free1)
