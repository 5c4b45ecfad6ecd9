"""Pins the CPU oracle against the reference's own known answers (tests/golden/reference_pins.json).

Every value below comes from an assertion in the reference's test suite (file:line in the JSON).
These run on CPU only; they are what makes the oracle trustworthy as the parity checker.
"""
import json
import math
from pathlib import Path

import numpy as np
import pytest

import oracle as orc

PINS = json.loads((Path(__file__).parent / "golden" / "reference_pins.json").read_text())


def test_rng_u64_streams():
    p = PINS["rng_u64"]
    for seed, key in ((0, "seed0"), (42, "seed42")):
        r = orc.Rng(seed)
        assert [r.next_u64() for _ in range(4)] == [int(x, 16) for x in p[key]]


def test_rng_below_and_next_f32():
    p = PINS["rng_below"]
    r = orc.Rng(p["seed"])
    assert [r.below(p["n"]) for _ in range(8)] == p["values"]
    p = PINS["rng_next_f32"]
    r = orc.Rng(p["seed"])
    for want in p["values"]:
        assert abs(r.next_f32() - want) < p["tol"]


def test_rng_normal_moments_and_shuffle_is_a_permutation():
    # rng.rs:168-177 and :195-207
    r = orc.Rng(2024)
    s = np.array([r.normal() for _ in range(200_000)], np.float64)
    assert abs(s.mean()) < 0.01 and abs(s.var() - 1.0) < 0.02
    a = orc.Rng(3).shuffle(np.arange(50))
    b = orc.Rng(4).shuffle(np.arange(50))
    assert sorted(a.tolist()) == list(range(50)) and a.tolist() != list(range(50)) and a.tolist() != b.tolist()


def test_preset_parameter_counts():
    p = PINS["preset_params"]
    for name in orc.PRESETS:
        assert orc.param_breakdown(orc.preset(name))["total"] == p[name], name


def test_smoke_breakdown_untied_and_grouped():
    p = PINS["smoke_breakdown"]
    b = orc.param_breakdown(orc.preset("smoke"))
    for k in ("embedding", "attention", "mlp", "norms", "lm_head", "total"):
        assert b[k] == p[k], k
    cfg = orc.preset("smoke")
    cfg[9] = 0
    assert orc.param_breakdown(cfg)["total"] == p["untied_total"]
    cfg = orc.preset("smoke")
    cfg[4] = 1
    assert orc.param_breakdown(cfg)["attention"] == p["gqa1_attention"]


@pytest.mark.parametrize("field,index,value", [
    ("vocab_size", 0, 0), ("n_heads", 1, 63), ("n_kv_heads", 4, 3), ("d_model", 1, 60),
    ("rope_theta", 7, float("nan")), ("norm_eps", 8, 0.0), ("max_seq_len", 6, 0)])
def test_validation_names_the_offending_field(field, index, value):
    # config.rs:236-260
    cfg = orc.preset("smoke")
    cfg[index] = value
    with pytest.raises(ValueError, match=field):
        orc.param_breakdown(cfg)


def test_gemm_hand_calculation_and_matmul_gradients():
    p = PINS["gemm_hand"]
    a, b = np.array(p["a"], np.float32), np.array(p["b"], np.float32)
    np.testing.assert_array_equal(orc.gemm_nn(a, b), p["c"])
    np.testing.assert_array_equal(orc.gemm_nt(a, b.T.copy()), p["c"])
    np.testing.assert_array_equal(orc.gemm_tn(a.T.copy(), b), p["c"])
    g = PINS["matmul_grads"]
    ones = np.ones((2, 2), np.float32)
    np.testing.assert_array_equal(orc.gemm_nt(ones, b).ravel(), g["da"])
    np.testing.assert_array_equal(orc.gemm_tn(a, ones).ravel(), g["db"])


def test_gemm_nt_sums_in_ascending_inner_order():
    # ops_matmul.rs:263-276: 1e8 added last keeps nothing of the ones before it
    k = 40
    a = np.ones((1, k), np.float32)
    a[0, -1] = 1e8
    want = np.float32(0)
    for v in a[0]:
        want = np.float32(want + v)
    assert orc.gemm_nt(a, np.ones((1, k), np.float32))[0, 0] == want


def test_softmax_and_cross_entropy_known_values():
    p = PINS["softmax"]
    y = orc.softmax_rows(np.array([p["x"], [0, 0, 0]], np.float32))
    np.testing.assert_allclose(y[0], p["y"], atol=p["tol"])
    np.testing.assert_allclose(y[1], [1 / 3] * 3, atol=p["tol"])
    c = PINS["cross_entropy"]
    assert abs(orc.cross_entropy([[0.0, 0.0]], [0]) - c["uniform2_loss"]) < c["tol"]
    assert orc.cross_entropy([[20.0, 0.0, 0.0]], [0]) < 1e-6
    assert abs(orc.cross_entropy([[0.0, 0.0], [50.0, -50.0]], [1, 0]) - c["two_rows_loss"]) < c["tol"]
    _, g = orc.cross_entropy([[0.0, 0.0]], [0], grad=True)
    np.testing.assert_allclose(g[0], c["grad_uniform2_target0"], atol=c["tol"])
    big = orc.softmax_rows(np.array([[1000.0, 1000.0, -1000.0]], np.float32))
    np.testing.assert_allclose(big[0], [0.5, 0.5, 0.0], atol=1e-6)


def test_attention_known_answer_and_weights():
    p = PINS["attention_known"]
    q = np.array(p["q"], np.float32).reshape(1, 1, 2, 4)
    k = np.array(p["k"], np.float32).reshape(1, 1, 2, 4)
    v = np.array(p["v"], np.float32).reshape(1, 1, 2, 4)
    out, probs = orc.causal_attention(q, k, v, 1, 1)
    w0 = 1.0 / (1.0 + math.exp(-1.0))
    np.testing.assert_allclose(out.ravel(), [1, 0, 0, 0, w0, 1 - w0, 0, 0], atol=p["tol"])
    np.testing.assert_allclose(probs.ravel(), [1, 0, w0, 1 - w0], atol=p["tol"])


def test_attention_rows_are_causal_distributions_and_groups_share_keys():
    # attention.rs:340-371
    rng = np.random.default_rng(0)
    q = rng.uniform(-1, 1, (2, 4, 5, 4)).astype(np.float32)
    k = rng.uniform(-1, 1, (2, 2, 5, 4)).astype(np.float32)
    v = rng.uniform(-1, 1, (2, 2, 5, 4)).astype(np.float32)
    _, probs = orc.causal_attention(q, k, v, 4, 2)
    for row_i in range(5):
        rows = probs[:, :, row_i, :]
        np.testing.assert_allclose(rows.sum(-1), 1.0, atol=1e-5)
        assert (rows[..., row_i + 1:] == 0).all() and (rows[..., :row_i + 1] > 0).all()
    q_same = np.repeat(q[:, :1], 4, axis=1)
    _, p2 = orc.causal_attention(q_same, k, v, 4, 2)
    np.testing.assert_array_equal(p2[:, 0], p2[:, 1])
    assert not np.array_equal(p2[:, 0], p2[:, 2])


def test_rope_table_formula():
    p = PINS["rope_table"]
    cos, sin = orc.rope_table(p["head_dim"], p["max_seq_len"], p["theta"])
    assert abs(cos[3, 0] - math.cos(3)) < p["tol"] and abs(sin[3, 0] - math.sin(3)) < p["tol"]
    assert abs(cos[3, 1] - math.cos(0.03)) < p["tol"] and abs(sin[3, 1] - math.sin(0.03)) < p["tol"]
    cos, sin = orc.rope_table(6, 9, 10000.0)
    np.testing.assert_array_equal(cos[0], [1, 1, 1])
    np.testing.assert_array_equal(sin[0], [0, 0, 0])
    np.testing.assert_allclose(cos * cos + sin * sin, 1.0, atol=1e-6)


def test_adamw_three_steps_and_decay_only():
    p = PINS["adamw_three_steps"]
    w = np.array(p["w0"], np.float32)
    b = np.array(p["b0"], np.float32)
    mw, vw, mb, vb = (np.zeros_like(w), np.zeros_like(w), np.zeros_like(b), np.zeros_like(b))
    b1, b2 = p["betas"]
    for step, ((lr, gw, gb), (want_w, want_b)) in enumerate(zip(p["steps"], p["after"]), start=1):
        orc.adamw_update(w, gw, mw, vw, True, step, lr, b1, b2, p["eps"], p["weight_decay"])
        orc.adamw_update(b, gb, mb, vb, False, step, lr, b1, b2, p["eps"], p["weight_decay"])
        np.testing.assert_allclose(w, want_w, atol=p["tol"])
        np.testing.assert_allclose(b, want_b, atol=p["tol"])
    d = PINS["adamw_decay_only"]
    w = np.array(p["w0"], np.float32)
    b = np.array(p["b0"], np.float32)
    z = np.zeros_like
    orc.adamw_update(w, z(w), z(w), z(w), True, 1, d["lr"], *d["betas"], 1e-8, d["weight_decay"])
    orc.adamw_update(b, z(b), z(b), z(b), False, 1, d["lr"], *d["betas"], 1e-8, d["weight_decay"])
    np.testing.assert_allclose(w, d["w_after"], atol=d["tol"])
    np.testing.assert_array_equal(b, np.array(d["b_after"], np.float32))


def test_schedule_values():
    p = PINS["schedule"]
    for step, want in p["values"]:
        assert abs(orc.schedule_lr(p["max_lr"], p["min_lr"], p["warmup"], p["total"], step) - want) < p["tol"]
    p = PINS["schedule_training_config"]
    for step, want in p["values"]:
        assert orc.schedule_lr(p["max_lr"], p["min_lr"], p["warmup"], p["total"], step) == np.float32(want)


def test_clip_norm_spans_every_gradient_and_refuses_non_finite():
    g = np.array([3.0, 0.0, 4.0], np.float32)
    norm, ok = orc.clip_global_norm(g.copy(), 10.0)
    assert ok and abs(norm - PINS["clip_norm"]["norm"]) < 1e-6
    clipped = g.copy()
    norm, ok = orc.clip_global_norm(clipped, 1.0)
    assert ok and abs(np.linalg.norm(clipped) - 1.0) < 1e-5
    bad = np.array([1.0, np.inf], np.float32)
    _, ok = orc.clip_global_norm(bad, 1.0)
    assert not ok and bad[0] == 1.0


def test_batch_windows_counts_and_epoch_order():
    p = PINS["batch_windows"]
    b = orc.Batcher(np.arange(21), 4, 1, 7)
    assert len(b) == 5
    seen = {}
    for _ in range(5):
        i, t, epoch, _idx = b.next()
        seen[int(i[0]) // 4] = list(i) + [int(t[-1])]
        assert epoch == 0
    assert [seen[k] for k in range(5)] == p["windows_21_4"]
    for tokens, count in p["counts_seq4"]:
        if count == 0:
            continue
        assert len(orc.Batcher(np.arange(tokens), 4, 1, 0)) == count
    assert len(orc.Batcher(np.arange(10), 1, 1, 0)) == p["count_10_seq1"]
    # the order of each pass is Rng(seed).fork(epoch).shuffle(0..n) (batch.rs:244-248)
    n, seed = 10, 7
    tok = np.arange(n * 4 + 1)
    b = orc.Batcher(tok, 4, 3, seed)
    for epoch in range(3):
        order = orc.Rng(seed).fork(epoch).shuffle(np.arange(n))
        for k in range(n // 3):
            i, _, e, idx = b.next()
            assert (e, idx) == (epoch, k)
            assert [int(x) // 4 for x in i[::4]] == [int(s) for s in order[3 * k:3 * k + 3]]


WIRING = PINS["wiring_config"]


def wiring_cfg(tie):
    w = WIRING
    return orc.config_array(w["vocab"], w["d_model"], w["n_layers"], w["n_heads"], w["n_kv_heads"], w["d_ff"],
                            w["max_seq_len"], tie=tie)


def test_parameter_names_order_and_accounting():
    m = orc.Model(wiring_cfg(False), seed=0)
    names = [t[0] for t in m.tensors()]
    assert names[0] == "embed_tokens.weight" and names[1] == "blocks.0.attn_norm.weight"
    assert names[-3] == "blocks.2.mlp.down_proj.weight" and names[-2] == "final_norm.weight"
    assert names[-1] == "lm_head.weight" and len(names) == 30 and len(set(names)) == 30
    assert m.n == orc.param_breakdown(wiring_cfg(False))["total"]


def test_init_draws_the_documented_standard_deviations():
    p = PINS["init_std"]
    cfg = wiring_cfg(False)
    m = orc.Model(cfg, seed=p["seed"], init_std=p["std"])
    params = m.params
    residual = p["std"] / math.sqrt(2.0 * WIRING["n_layers"])
    for name, _shape, off, n in m.tensors():
        x = params[off:off + n]
        rms = float(np.sqrt((x.astype(np.float64) ** 2).mean()))
        want = 1.0 if name.endswith("_norm.weight") else (
            residual if name.endswith(("o_proj.weight", "down_proj.weight")) else p["std"])
        assert abs(rms - want) < p["slack"] * want, name


def test_one_seed_fixes_the_model_and_causality_holds():
    ids = np.array([1, 4, 2, 7, 3, 9], np.int32)
    a = orc.Model(wiring_cfg(True), seed=5).logits(ids, 1, 6)
    b = orc.Model(wiring_cfg(True), seed=5).logits(ids, 1, 6)
    c = orc.Model(wiring_cfg(True), seed=6).logits(ids, 1, 6)
    np.testing.assert_array_equal(a, b)
    assert not np.array_equal(a, c)
    m = orc.Model(wiring_cfg(True), seed=1, init_std=0.3)
    base_ids = np.array([3, 1, 4, 1, 5, 9], np.int32)
    base = m.logits(base_ids, 1, 6)[0]
    for pos in range(1, 6):
        ids = base_ids.copy()
        ids[pos] = (ids[pos] + 1) % 13
        changed = m.logits(ids, 1, 6)[0]
        np.testing.assert_allclose(changed[:pos], base[:pos], atol=1e-5)
        assert not np.array_equal(changed[pos], base[pos])


def test_batch_loss_is_the_mean_of_sequence_losses():
    # wiring.rs:207-216
    m = orc.Model(wiring_cfg(False), seed=6, init_std=0.3)
    a, b = [1, 5, 2, 8, 3], [12, 0, 7, 7, 4]
    ta, tb = [5, 2, 8, 3, 6], [0, 7, 7, 4, 10]
    together = m.loss(a + b, ta + tb, 2, 5)
    assert abs(together - (m.loss(a, ta, 1, 5) + m.loss(b, tb, 1, 5)) / 2) < 1e-5


def test_fresh_model_loss_is_near_uniform():
    # model.rs:256-263
    cfg = orc.config_array(11, 8, 2, 2, 1, 12, 6)
    m = orc.Model(cfg, seed=1)
    loss = m.loss([0, 3, 5, 7, 2, 9], [3, 5, 7, 2, 9, 1], 2, 3)
    assert abs(loss - math.log(11)) < 0.15


def _fd_agreement(tie, batch, seq):
    p = PINS["fd_gradients"]
    cfg = wiring_cfg(tie)
    m = orc.Model(cfg, seed=p["model_seed"], init_std=p["init_std"])
    ids = orc.Rng(p["ids_seed"])
    inputs = [ids.below(13) for _ in range(batch * seq)]
    targets = [ids.below(13) for _ in range(batch * seq)]
    _, grads = m.loss(inputs, targets, batch, seq, grads=True)
    base = m.params
    pick = orc.Rng(p["pick_seed"])
    eps = np.float32(p["eps"])
    diff_sq = ref_sq = 0.0
    per = []
    for name, _shape, off, n in m.tensors():
        pd = pr = 0.0
        for _ in range(p["samples_per_param"]):
            at = off + pick.below(n)

            def loss_at(delta):
                x = base.copy()
                x[at] = np.float32(x[at] + delta)
                m.params = x
                return m.loss(inputs, targets, batch, seq)
            numeric = float(np.float32(loss_at(eps) - loss_at(-eps))) / (2.0 * float(eps))
            exact = float(grads[at])
            pd += (numeric - exact) ** 2
            pr += exact ** 2
        m.params = base
        diff_sq += pd
        ref_sq += pr
        per.append((name, math.sqrt(pd / max(pr, 1e-12)), math.sqrt(pr), math.sqrt(pd)))
    return math.sqrt(diff_sq / ref_sq), math.sqrt(ref_sq), per


@pytest.mark.parametrize("tie,batch,seq", [(True, 2, 5), (False, 2, 5), (True, 1, 8), (False, 3, 1)])
def test_analytic_gradients_match_finite_differences(tie, batch, seq):
    # wiring.rs:294-336: the oracle's backward pass against central differences of its forward pass
    p = PINS["fd_gradients"]
    rel, size, per = _fd_agreement(tie, batch, seq)
    assert size > 1e-2
    assert rel < p["overall_max"], rel
    for name, err, psize, absolute in per:
        if seq == 1 and name.endswith(("q_proj.weight", "k_proj.weight")):
            assert psize == 0.0 and absolute < 1e-3, name
            continue
        assert psize > 1e-3, name
        assert err < p["per_param_max"], (name, err)
