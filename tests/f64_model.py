"""The MidMan decoder's loss and gradients in float64 PyTorch, as a third opinion.

Test infrastructure: at the benchmarked shapes the reference's own f32 arithmetic
(restated by the oracle) drifts from exact math by more than the 3xTF32 gate, so the
parity tests there also compare both the GPU step and the oracle with this float64
evaluation of the same model, weights and ids. It follows the reference's formulas,
not its operation order: crates/midman-model/src/model.rs:127-165 (embedding, blocks,
final RMSNorm, tied head), crates/midman-nn/src/block.rs:77-81 (pre-norm residual
blocks), norm.rs:21-39, rope.rs:20-33 (rotate-half with the f32 tables the reference
builds), attention.rs:79-102 (grouped heads, causal mask, scale 1/sqrt(hd) in f32),
mlp.rs:20-24 (SwiGLU) and ops_reduce.rs:236-276 (mean cross-entropy).
"""
import numpy as np


def loss_and_grads(torch, cfg, tensors, params, inputs, targets, batch, seq, cos_t, sin_t, device="cuda"):
    """cfg: the oracle's config array; tensors: [(name, shape, offset, numel)]; cos_t/sin_t: [seq, hd/2]
    f32 tables. Returns (loss, flat float64 gradient as numpy) in the order of `tensors`."""
    V, D, L, H, Hkv, F = (int(cfg[i]) for i in range(6))
    eps = float(np.float32(cfg[8]))
    hd = D // H
    G = H // Hkv
    flat = torch.tensor(params, dtype=torch.float64, device=device)
    w = {}
    for name, shape, off, n in tensors:
        w[name] = flat[off:off + n].view(*shape).clone().requires_grad_()
    ids = torch.tensor(np.asarray(inputs, np.int64), device=device)
    tgt = torch.tensor(np.asarray(targets, np.int64), device=device)
    cos = torch.tensor(cos_t[:seq], dtype=torch.float64, device=device)[None, :, None, :]
    sin = torch.tensor(sin_t[:seq], dtype=torch.float64, device=device)[None, :, None, :]
    scale = float(np.float32(1.0) / np.sqrt(np.float32(hd)))
    mask = torch.triu(torch.ones(seq, seq, dtype=torch.bool, device=device), 1)

    def rms(x, weight):
        return x * torch.rsqrt((x * x).mean(-1, keepdim=True) + eps) * weight

    def rope(x):  # [B, T, heads, hd]
        x1, x2 = x[..., :hd // 2], x[..., hd // 2:]
        return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], -1)

    x = w["embed_tokens.weight"][ids].view(batch, seq, D)
    for l in range(L):
        p = f"blocks.{l}."
        xn = rms(x, w[p + "attn_norm.weight"])
        q = rope((xn @ w[p + "attn.q_proj.weight"]).view(batch, seq, H, hd)).transpose(1, 2)
        k = rope((xn @ w[p + "attn.k_proj.weight"]).view(batch, seq, Hkv, hd)).transpose(1, 2)
        v = (xn @ w[p + "attn.v_proj.weight"]).view(batch, seq, Hkv, hd).transpose(1, 2)
        k = k.repeat_interleave(G, dim=1)
        v = v.repeat_interleave(G, dim=1)
        s = (q @ k.transpose(-1, -2)) * scale
        s = s.masked_fill(mask, float("-inf"))
        o = (torch.softmax(s, -1) @ v).transpose(1, 2).reshape(batch, seq, D)
        h = x + o @ w[p + "attn.o_proj.weight"]
        xn2 = rms(h, w[p + "mlp_norm.weight"])
        g = xn2 @ w[p + "mlp.gate_proj.weight"]
        u = xn2 @ w[p + "mlp.up_proj.weight"]
        x = h + (torch.nn.functional.silu(g) * u) @ w[p + "mlp.down_proj.weight"]
    xf = rms(x, w["final_norm.weight"])
    head = w["embed_tokens.weight"].t() if "lm_head.weight" not in w else w["lm_head.weight"]
    logits = (xf @ head).view(batch * seq, V)
    loss = torch.nn.functional.cross_entropy(logits, tgt)
    loss.backward()
    grads = torch.cat([w[name].grad.reshape(-1) for name, _s, _o, _n in tensors])
    return float(loss.item()), grads.cpu().numpy()
