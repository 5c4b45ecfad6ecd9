"""Causal grouped-query attention kernels (mm_gpu_attention_*) against float64 PyTorch.

The reference computes softmax(q k^T / sqrt(hd) + mask(-1e9)) v with grouped heads
expanded by copying (crates/midman-nn/src/attention.rs:79-102); its backward is the
autograd of that chain. MM_GPU_TF32 runs the score/value products on the tensor cores
in the fused flash kernels (relative L2 within 5e-3), MM_GPU_3XTF32 as three-term TF32
products on the tensor cores through score buffers (within 1e-5); head_dim 16 runs the
FP32 flash kernels in both.
"""
import math

import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

CASES = [  # (B, T, H, Hkv, hd)
    (2, 300, 4, 1, 32),
    (1, 130, 4, 2, 64),
    (2, 256, 2, 2, 128),
    (1, 64, 2, 1, 16),
    (1, 2048, 4, 2, 128),
    (3, 77, 6, 3, 64),
    (8, 1024, 16, 16, 64),  # configs[2]: B 8, 16 heads of 64, T 1024
    (4, 2048, 16, 8, 128),  # the attention of configs[4]'s layers: 512 query tiles over the persistent pairs
]


def reference(q, k, v, H, Hkv):
    """float64 attention on [B, T, heads, hd] inputs; returns o [B, T, H, hd] and lse [B, H, T]."""
    B, T, _, hd = q.shape
    G = H // Hkv
    qh = q.permute(0, 2, 1, 3)
    kh = k.permute(0, 2, 1, 3).repeat_interleave(G, dim=1)
    vh = v.permute(0, 2, 1, 3).repeat_interleave(G, dim=1)
    s = qh @ kh.transpose(-1, -2) / math.sqrt(hd)
    mask = torch.triu(torch.ones(T, T, dtype=torch.bool, device=q.device), 1)
    s = s.masked_fill(mask, float("-inf"))
    lse = torch.logsumexp(s, -1)
    o = torch.softmax(s, -1) @ vh
    return o.permute(0, 2, 1, 3), lse


def rel(a, b):
    return ((a.double() - b).norm() / b.norm()).item()


@pytest.mark.parametrize("precision", [0, 1])
@pytest.mark.parametrize("case", CASES)
def test_attention_forward_and_backward(mm, case, precision):
    B, T, H, Hkv, hd = case
    g = torch.Generator(device="cuda").manual_seed(B * 1000 + T)
    D, KV = H * hd, Hkv * hd
    q = torch.randn(B, T, H, hd, device="cuda", generator=g)
    k = torch.randn(B, T, Hkv, hd, device="cuda", generator=g)
    v = torch.randn(B, T, Hkv, hd, device="cuda", generator=g)
    do = torch.randn(B, T, H, hd, device="cuda", generator=g)
    o = torch.empty(B, T, H, hd, device="cuda")
    lse = torch.empty(B, H, T, device="cuda")
    kw = dict(batch=B, seq=T, n_heads=H, n_kv_heads=Hkv, head_dim=hd, ldq=D, ldk=KV, precision=precision)
    mm.attention_forward(q, k, v, o, lse, **kw)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    mm.attention_backward(q, k, v, o, lse, do, dq, dk, dv, **kw)
    mm.device_status()
    q64, k64, v64 = (x.double().requires_grad_() for x in (q, k, v))
    ro, rlse = reference(q64, k64, v64, H, Hkv)
    ro.backward(do.double())
    tol = 5e-3 if precision == 0 else 1e-5
    assert rel(o, ro.detach()) < tol
    assert (lse.double() - rlse.detach()).abs().max().item() < (1e-2 if precision == 0 else 1e-5)
    assert rel(dq, q64.grad) < tol
    assert rel(dk, k64.grad) < tol
    assert rel(dv, v64.grad) < tol
