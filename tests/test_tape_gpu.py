"""Device tensors with a recording autograd tape (include/midman_tensor.h).

The reference's midman-tensor records a node per operation whose inputs track
gradients and replays the nodes in reverse on Tensor::backward, summing the
gradients that reach a tensor from several uses (crates/midman-tensor/src/
autograd.rs:27-124). These tests drive the same API on the GPU: small graphs
against float64 PyTorch autograd (a tensor used several times, unused inputs,
leaves that do not track gradients), and the whole MidManModel built op by op
on the tape (model.rs:127-165) against the oracle's loss and per-tensor
gradients, with the gates of test_model_gpu.py (1e-5 in 3xTF32, 1e-2 in TF32).
"""
import math

import numpy as np
import pytest

import oracle as orc

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.fixture()
def tape(mm):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    t = mm.Tape(precision=1)
    yield t
    t.close()


def test_reused_tensors_sum_their_gradients(mm, tape):
    rs = np.random.default_rng(0)
    a = rs.standard_normal((6, 8)).astype(np.float32)
    b = rs.standard_normal((8, 12)).astype(np.float32)
    w = rs.standard_normal((12, 16)).astype(np.float32)
    c0 = rs.standard_normal((6, 12)).astype(np.float32)
    tgt = np.array([1, 3, 5, 7, 9, 11], np.int32)
    ta, tb, tw = (tape.tensor(x, requires_grad=True) for x in (a, b, w))
    tc0 = tape.tensor(c0)  # a constant: no gradient
    c = tape.matmul(ta, tb)                       # [6, 12]
    d = tape.add(tape.mul(c, c), tape.mul(c, tc0))  # c used three times
    e = tape.matmul(d, tw)                        # [6, 16]
    loss = tape.cross_entropy(e, tgt)
    tape.backward(loss)
    A, B, W = (torch.tensor(x, dtype=torch.float64, requires_grad=True) for x in (a, b, w))
    C = A @ B
    D = C * C + C * torch.tensor(c0, dtype=torch.float64)
    L = torch.nn.functional.cross_entropy(D @ W, torch.tensor(tgt, dtype=torch.long))
    L.backward()
    assert abs(tape.read(loss)[0] - L.item()) <= 1e-5 * abs(L.item())
    assert rel(tape.grad(ta), A.grad) < 1e-5
    assert rel(tape.grad(tb), B.grad) < 1e-5
    assert rel(tape.grad(tw), W.grad) < 1e-5
    assert not tape.grad(tc0).any()  # a constant gets no gradient
    # a second backward over a new graph replaces the gradients
    loss2 = tape.cross_entropy(tape.matmul(ta, tb), tgt)
    tape.backward(loss2)
    A2 = torch.tensor(a, dtype=torch.float64, requires_grad=True)
    torch.nn.functional.cross_entropy(A2 @ torch.tensor(b, dtype=torch.float64), torch.tensor(tgt,
                                                                                            dtype=torch.long)).backward()
    assert rel(tape.grad(ta), A2.grad) < 1e-5
    assert not tape.grad(tw).any()  # w is not in the second graph


def test_errors_are_status_codes(mm, tape):
    x = tape.tensor(np.ones((4, 6), np.float32), requires_grad=True)
    with pytest.raises(mm.MidmanGpuError, match="multiples of 4"):
        tape.matmul(x, tape.tensor(np.ones((6, 6), np.float32)))
    with pytest.raises(mm.MidmanGpuError, match="does not track"):
        tape.backward(tape.cross_entropy(tape.tensor(np.ones((2, 4), np.float32)), [0, 1]))
    table = tape.tensor(np.ones((5, 4), np.float32), requires_grad=True)
    with pytest.raises(mm.MidmanGpuError, match="outside"):
        tape.embedding(table, [0, 5])
    with pytest.raises(mm.MidmanGpuError, match="not live"):
        tape.read(12345)


def model_on_tape(tape, cfg, params, tensors, inputs, targets, B, T):
    """MidManModel::run (model.rs:127-165) and the loss, op by op on the tape."""
    V, D, L, H, Hkv, F = (int(cfg[i]) for i in range(6))
    theta, eps = float(cfg[7]), float(np.float32(cfg[8]))
    hd = D // H
    w = {name: tape.tensor(params[off:off + n].reshape(shape), requires_grad=True)
         for name, shape, off, n in tensors}
    x = tape.embedding(w["embed_tokens.weight"], inputs)
    for l in range(L):
        p = f"blocks.{l}."
        xn = tape.rms_norm(x, w[p + "attn_norm.weight"], eps)
        q = tape.rope(tape.matmul(xn, w[p + "attn.q_proj.weight"]), T, H, theta)
        k = tape.rope(tape.matmul(xn, w[p + "attn.k_proj.weight"]), T, Hkv, theta)
        v = tape.matmul(xn, w[p + "attn.v_proj.weight"])
        o = tape.causal_attention(q, k, v, B, T, H, Hkv)
        h = tape.add(x, tape.matmul(o, w[p + "attn.o_proj.weight"]))
        xn2 = tape.rms_norm(h, w[p + "mlp_norm.weight"], eps)
        act = tape.swiglu(tape.matmul(xn2, w[p + "mlp.gate_proj.weight"]),
                          tape.matmul(xn2, w[p + "mlp.up_proj.weight"]))
        x = tape.add(h, tape.matmul(act, w[p + "mlp.down_proj.weight"]))
    xf = tape.rms_norm(x, w["final_norm.weight"], eps)
    if "lm_head.weight" in w:
        logits = tape.matmul(xf, w["lm_head.weight"])
    else:
        logits = tape.matmul(xf, w["embed_tokens.weight"], b_transposed=True)  # x E^T, tied
    loss = tape.cross_entropy(logits, targets)
    tape.backward(loss)
    return float(tape.read(loss)[0]), {name: tape.grad(t).ravel() for name, t in w.items()}


MODELS = {
    "gqa_small": (orc.config_array(64, 32, 2, 4, 2, 48, 16), 2, 16, 0.3),
    "untied": (orc.config_array(64, 32, 2, 4, 2, 48, 16, tie=False), 2, 16, 0.3),
    "hd64_T130": (orc.config_array(96, 256, 2, 4, 2, 128, 130), 1, 130, 0.05),
    "tiny_preset": (orc.preset("tiny"), 2, 128, 0.02),
}


@pytest.mark.parametrize("precision", [1, 0])
@pytest.mark.parametrize("case", list(MODELS))
def test_the_model_built_on_the_tape_matches_the_oracle(mm, case, precision):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    cfg, B, T, std = MODELS[case]
    model = orc.Model(cfg, seed=31, init_std=std)
    r = orc.Rng(32)
    inputs = np.array([r.below(int(cfg[0])) for _ in range(B * T)], np.int32)
    targets = np.array([r.below(int(cfg[0])) for _ in range(B * T)], np.int32)
    want_loss, want_g = model.loss(inputs, targets, B, T, grads=True)
    tape = mm.Tape(precision=precision)
    try:
        loss, grads = model_on_tape(tape, cfg, model.params, model.tensors(), inputs, targets, B, T)
    finally:
        tape.close()
    tol = 1e-5 if precision == 1 else 1e-2
    assert abs(loss - want_loss) <= (1e-6 if precision == 1 else 1e-3) * max(1.0, abs(want_loss)), (loss, want_loss)
    worst = max((rel(grads[name], want_g[off:off + n]), name) for name, _s, off, n in model.tensors())
    assert worst[0] <= tol, worst
    assert math.isfinite(loss)
