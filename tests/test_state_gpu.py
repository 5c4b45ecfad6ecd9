"""Training-state files (midman_train_save / midman_train_restore) on the GPU.

The state file of crates/midman-training/src/state.rs:45-288: the library writes
the reference's bytes (checked against oracle/safetensors.py, the Python
restatement of the reference writer), a run restored from it continues
bit-for-bit, a refused load changes nothing (state.rs:412-488), and a state moves
between the CPU oracle and the GPU in both directions (the resume property of
tests/resume.rs in the reference, here across devices).
"""
import struct

import numpy as np
import pytest

import oracle as orc
import safetensors as st

pytestmark = pytest.mark.gpu

ERR_ARGUMENT, ERR_SHAPE, ERR_OTHER = -1, -3, -5
CFG = orc.config_array(64, 32, 2, 4, 2, 48, 16)
B, T = 2, 16
HYPER = dict(max_lr=0.02, min_lr=0.002, warmup=2, total=40, weight_decay=0.1, clip_norm=1.0, beta1=0.9, beta2=0.95)


def batches(seed, n):
    r = orc.Rng(seed)
    out = []
    for _ in range(n):
        ids = np.array([r.below(64) for _ in range(B * (T + 1))], np.int32).reshape(B, T + 1)
        out.append((ids[:, :T].ravel().copy(), ids[:, 1:].ravel().copy()))
    return out


def trainer(mm, seed=3, **hyper_over):
    h = dict(HYPER, **hyper_over)
    return mm.Trainer(CFG, mm.hyper_array(**h), seed=seed, batch=B, seq=T, precision=1)


def names_shapes():
    return [(n, s) for n, s, _off, _num in orc.Model(CFG, seed=0).tensors()]


def tensors_of(t, which):
    return [(n, s, t.read(which, i)) for i, (n, s) in enumerate(names_shapes())]


def settings(seed=5, **over):
    h = dict(HYPER, **over)
    return st.settings_metadata(B, T, seed, h["max_lr"], h["min_lr"], h["warmup"], h["total"], h["beta1"],
                                h["beta2"], 1e-8, h["weight_decay"], h["clip_norm"])


def bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


def test_the_saved_file_is_the_reference_state_file(mm, tmp_path):
    t = trainer(mm)
    for i, (x, y) in enumerate(batches(11, 3)):
        _, status = t.step(x, y)
        assert status == 0
    path = tmp_path / "state.safetensors"
    t.save(path, data_seed=5, epoch=1, position=3)
    params = tensors_of(t, 0)
    moments = [(n, m, v) for (n, _s, m), (_n, _s2, v) in zip(tensors_of(t, 2), tensors_of(t, 3))]
    want = st.state_bytes(params, moments, step=3, epoch=1, position=3, settings=settings())
    assert path.read_bytes() == want
    info = mm.state_inspect(path)
    assert info["progress"] == {"step": 3, "epoch": 1, "position": 3}
    assert info["metadata"]["train.eps"] == "0.00000001" and info["metadata"]["train.max_lr"] == "0.02"
    # before the first step there are no moments (state.rs:487-505)
    fresh = trainer(mm)
    fresh.save(tmp_path / "zero.safetensors")
    names = [x["name"] for x in mm.state_inspect(tmp_path / "zero.safetensors")["tensors"]]
    assert names and all(n.startswith("param/") for n in names)
    t.close()
    fresh.close()


def test_a_restored_run_continues_bit_for_bit(mm, tmp_path):
    data = batches(12, 5)
    a = trainer(mm, seed=3)
    for x, y in data[:3]:
        a.step(x, y)
    path = tmp_path / "s.safetensors"
    a.save(path, data_seed=5, epoch=0, position=3)
    b = trainer(mm, seed=99)  # another init
    assert b.restore(path, data_seed=5) == {"step": 3, "epoch": 0, "position": 3}
    for which in (0, 2, 3):
        assert np.array_equal(bits(a.read(which)), bits(b.read(which)))
    for x, y in data[3:]:
        ra, sa = a.step(x, y)
        rb, sb = b.step(x, y)
        assert sa == sb == 0 and np.array_equal(bits(ra), bits(rb))
    assert np.array_equal(bits(a.params()), bits(b.params()))
    a.close()
    b.close()


def test_a_refused_restore_changes_nothing(mm, tmp_path):
    a = trainer(mm, seed=3)
    for x, y in batches(13, 2):
        a.step(x, y)
    good = tmp_path / "good.safetensors"
    a.save(good, data_seed=5)
    params = tensors_of(a, 0)
    moments = [(n, m, v) for (n, _s, m), (_n, _s2, v) in zip(tensors_of(a, 2), tensors_of(a, 3))]

    shapes = dict(names_shapes())

    def variant(name, params=params, moments=moments, **md):
        """The good state with some tensors or metadata entries changed."""
        meta = settings()
        meta.update(format="midman-training-state", state_version="1", step="2", epoch="0", position="0")
        meta.update(md)
        tensors = [("param/" + n, sh, v) for n, sh, v in params]
        for n, m, v in moments:
            tensors += [("adamw.m/" + n, shapes[n], m), ("adamw.v/" + n, shapes[n], v)]
        p = tmp_path / name
        p.write_bytes(st.to_bytes(tensors, meta))
        return p

    neg_v = [(n, m, (-np.abs(v) - 1.0) if i == 0 else v) for i, (n, m, v) in enumerate(moments)]
    wrong_shape = [(n, (s[0] * s[1],) if i == 0 else s, v) for i, (n, s, v) in enumerate(params)]  # embedding flat
    cases = [
        ("other settings", variant("lr.safetensors", **{"train.max_lr": "0.5"}), ERR_ARGUMENT, "train.max_lr"),
        ("no parameter", variant("np.safetensors", params=params[1:]), ERR_ARGUMENT, "missing"),
        ("a tensor nobody wants", variant("x.safetensors", params=params + [("extra", (1,), np.zeros(1, np.float32))]),
         ERR_ARGUMENT, "param/extra"),
        ("negative second moment", variant("v.safetensors", moments=neg_v), ERR_ARGUMENT, "second moment"),
        ("another shape", variant("sh.safetensors", params=wrong_shape), ERR_SHAPE, "shape"),
        ("another format", variant("f.safetensors", format="something-else"), ERR_OTHER, "something-else"),
        ("another version", variant("ver.safetensors", state_version="2"), ERR_OTHER, "version"),
    ]
    b = trainer(mm, seed=99)
    before = [b.read(w) for w in (0, 2, 3)]
    for what, path, status, mention in cases:
        with pytest.raises(mm.MidmanError) as e:
            b.restore(path, data_seed=5)
        assert e.value.status == status, (what, e.value)
        assert mention in e.value.message, (what, e.value.message)
        for w, old in zip((0, 2, 3), before):
            assert np.array_equal(bits(b.read(w)), bits(old)), what
    with pytest.raises(mm.MidmanError) as e:  # the data seed is a setting of the run too
        b.restore(good, data_seed=6)
    assert "train.seed" in e.value.message
    assert b.restore(good, data_seed=5)["step"] == 2
    a.close()
    b.close()


def read_state(mm, path):
    """Flat params / m / v of a state file, through the library's checked header."""
    info = mm.state_inspect(path)
    raw = path.read_bytes()
    off = 8 + struct.unpack("<Q", raw[:8])[0]
    by_name = {t["name"]: np.frombuffer(raw[off + t["data_offsets"][0]: off + t["data_offsets"][1]], "<f4")
               for t in info["tensors"]}
    model_names = [n for n, _ in names_shapes()]
    flat = lambda prefix: np.concatenate([by_name[prefix + n] for n in model_names]) if (prefix + model_names[0]) in by_name else None
    return info["progress"], flat("param/"), flat("adamw.m/"), flat("adamw.v/")


def test_a_state_moves_between_the_cpu_oracle_and_the_gpu(mm, tmp_path):
    data = batches(14, 4)
    model = orc.Model(CFG, seed=3)
    opt = orc.AdamW(model, HYPER["beta1"], HYPER["beta2"], 1e-8, HYPER["weight_decay"])
    sched = lambda s: orc.schedule_lr(HYPER["max_lr"], HYPER["min_lr"], HYPER["warmup"], HYPER["total"], s)
    for step, (x, y) in enumerate(data[:2]):
        assert orc.train_update(model, opt, x, y, B, T, HYPER["clip_norm"], sched(step))[2]
    # the CPU run's state, written as the reference writes it
    m, v = opt.moments()
    tensors = [(n, s, model.params[o:o + c]) for n, s, o, c in model.tensors()]
    moments = [(n, m[o:o + c], v[o:o + c]) for n, s, o, c in model.tensors()]
    cpu_file = tmp_path / "cpu.safetensors"
    cpu_file.write_bytes(st.state_bytes(tensors, moments, step=2, epoch=0, position=2, settings=settings()))
    g = trainer(mm, seed=77)
    assert g.restore(cpu_file, data_seed=5)["step"] == 2
    assert np.array_equal(bits(g.params()), bits(model.params))
    # one step on each side from the same state (3xTF32 against the f32 oracle)
    x, y = data[2]
    rec, status = g.step(x, y)
    loss, norm, ok = orc.train_update(model, opt, x, y, B, T, HYPER["clip_norm"], sched(2))
    assert status == 0 and ok
    assert abs(rec[0] - loss) <= 1e-5 * abs(loss) and abs(rec[1] - norm) <= 1e-4 * abs(norm)
    p_gpu, p_cpu = g.params(), model.params
    assert np.linalg.norm(p_gpu - p_cpu) <= 1e-5 * np.linalg.norm(p_cpu)
    # and back: the GPU's state into a fresh oracle run
    gpu_file = tmp_path / "gpu.safetensors"
    g.save(gpu_file, data_seed=5, epoch=0, position=3)
    progress, p, m2, v2 = read_state(mm, gpu_file)
    assert progress["step"] == 3
    model2 = orc.Model(CFG, seed=1234)
    model2.params = p
    opt2 = orc.AdamW(model2, HYPER["beta1"], HYPER["beta2"], 1e-8, HYPER["weight_decay"])
    opt2.restore(progress["step"], m2, v2)
    x, y = data[3]
    loss2, _, ok2 = orc.train_update(model2, opt2, x, y, B, T, HYPER["clip_norm"], sched(3))
    rec2, status2 = g.step(x, y)
    assert ok2 and status2 == 0
    assert abs(rec2[0] - loss2) <= 1e-5 * abs(loss2)
    assert np.linalg.norm(g.params() - model2.params) <= 1e-5 * np.linalg.norm(model2.params)
    g.close()
