"""Training from token-shard files on the GPU (midman_train_run).

midman_train_run is the reference's training loop over a Batcher
(crates/midman-training/src/trainer.rs:162-183 fed by crates/midman-data/src/
batch.rs:113-248): the host takes and prepares the next batch while the GPU runs
the current step. Here it must give exactly the steps of taking each batch by
hand (midman_batcher_next + midman_train_step), put the batcher back when a batch
is refused, and continue bit-for-bit from a state file and a batcher seek (the
resume property of the reference's tests/resume.rs).
"""
import numpy as np
import pytest

import oracle as orc
import token_shard as ts

pytestmark = pytest.mark.gpu

CFG = orc.config_array(64, 32, 2, 4, 2, 48, 16)
B, T = 2, 16
HYPER = dict(max_lr=0.02, min_lr=0.002, warmup=2, total=40, weight_decay=0.1, clip_norm=1.0, beta1=0.9, beta2=0.95)


def trainer(mm, seed=3):
    return mm.Trainer(CFG, mm.hyper_array(**HYPER), seed=seed, batch=B, seq=T, precision=1)


def shards(tmp_path, lengths, vocab=64, seed=0, bad=None):
    """Shard files of random ids below `vocab`; `bad` = (shard, index, id) plants one id."""
    r = np.random.default_rng(seed)
    paths = []
    for k, n in enumerate(lengths):
        t = r.integers(0, 64, n).astype(np.uint32)
        if bad is not None and bad[0] == k:
            t[bad[1]] = bad[2]
        p = tmp_path / f"train-{k}.mmtokens"
        p.write_bytes(ts.to_bytes(vocab, 0, t))
        paths.append(p)
    return paths


def bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


def test_training_from_shards_equals_taking_each_batch_by_hand(mm, tmp_path):
    paths = shards(tmp_path, [200, 70, 15, 130])
    a, b = trainer(mm), trainer(mm)
    ba = mm.Batcher(shards=paths, seq=T, batch=B, seed=9)
    bb = mm.Batcher(shards=paths, seq=T, batch=B, seed=9)
    rec, status, place = a.run(ba, 14)  # more steps than an epoch: (12 + 4 + 0 + 8) windows / 2
    assert status == 0 and rec.shape == (14, 3)
    for s in range(14):
        x, y, _, _ = bb.next()
        r, st = b.step(x, y)
        assert st == 0 and np.array_equal(bits(r), bits(rec[s])), s
    assert np.array_equal(bits(a.params()), bits(b.params()))
    assert place == bb.seek(place["epoch"], place["position"])
    assert place["epoch"] == 1 and place["position"] == 2
    x1, y1, e1, i1 = ba.next()
    x2, y2, e2, i2 = bb.next()
    assert np.array_equal(x1, x2) and (e1, i1) == (e2, i2)
    for h in (a, b, ba, bb):
        h.close()


def test_a_refused_batch_leaves_the_batcher_before_it(mm, tmp_path):
    # a shard id of 63 < 100 is valid for the shard, 70 is not for a model of 64 ids
    lengths = [161, 97]
    paths = shards(tmp_path, lengths, vocab=100, seed=1, bad=(1, 40, 70))
    ref = orc.Batcher(np.concatenate([ts_tokens(p) for p in paths]), T, B, 5, shard_lengths=lengths)
    k = 0
    while True:
        i, t, _, _ = ref.next()
        if (i >= 64).any() or (t >= 64).any():
            break
        k += 1
    assert 0 < k < 20
    a = trainer(mm)
    batcher = mm.Batcher(shards=paths, seq=T, batch=B, seed=5)
    with pytest.raises(mm.MidmanError) as e:
        a.run(batcher, k + 5)
    assert "70" in e.value.message
    # k steps were taken; the batcher is back before the refused batch
    by_hand = trainer(mm)
    hand = mm.Batcher(shards=paths, seq=T, batch=B, seed=5)
    for _ in range(k):
        x, y, _, _ = hand.next()
        assert by_hand.step(x, y)[1] == 0
    assert np.array_equal(bits(a.params()), bits(by_hand.params()))
    got, want = batcher.next(), hand.next()
    assert np.array_equal(got[0], want[0]) and got[2:] == want[2:]
    for h in (a, by_hand, batcher, hand):
        h.close()


def ts_tokens(path):
    raw = path.read_bytes()
    width = int.from_bytes(raw[12:16], "little")
    return np.frombuffer(raw[32:-32], "<u2" if width == 2 else "<u4").astype(np.uint32)


def test_a_run_resumes_from_its_state_file_and_batcher_place(mm, tmp_path):
    paths = shards(tmp_path, [300, 111, 90], seed=2)
    cont = trainer(mm)
    cb = mm.Batcher(shards=paths, seq=T, batch=B, seed=21)
    rec1, st1, place = cont.run(cb, 4)
    assert st1 == 0
    path = tmp_path / "state.safetensors"
    cont.save(path, data_seed=21, epoch=place["epoch"], position=place["position"])
    rec2, st2, place2 = cont.run(cb, 5)
    resumed = trainer(mm, seed=1234)
    progress = resumed.restore(path, data_seed=21)
    assert progress == {"step": 4, "epoch": place["epoch"], "position": place["position"]}
    rb = mm.Batcher(shards=paths, seq=T, batch=B, seed=21)
    rb.seek(progress["epoch"], progress["position"])
    rec3, st3, place3 = resumed.run(rb, 5)
    assert st2 == st3 == 0 and place2 == place3
    assert np.array_equal(bits(rec2), bits(rec3))
    assert np.array_equal(bits(cont.params()), bits(resumed.params()))
    for h in (cont, cb, resumed, rb):
        h.close()


def test_zero_steps_take_no_batch(mm, tmp_path):
    paths = shards(tmp_path, [300], seed=6)
    t = trainer(mm)
    b = mm.Batcher(shards=paths, seq=T, batch=B, seed=1)
    rec, status, place = t.run(b, 0)
    assert status == 0 and rec.shape == (0, 3) and (place["epoch"], place["position"]) == (0, 0)
    fresh = mm.Batcher(shards=paths, seq=T, batch=B, seed=1)
    assert np.array_equal(b.next()[0], fresh.next()[0])
    for h in (t, b, fresh):
        h.close()


def test_the_batcher_must_fit_the_run(mm, tmp_path):
    paths = shards(tmp_path, [300], seed=3)
    t = trainer(mm)
    wrong = mm.Batcher(shards=paths, seq=T, batch=B + 1, seed=0)
    with pytest.raises(mm.MidmanError) as e:
        t.run(wrong, 1)
    assert e.value.status == -1
    fresh = mm.Batcher(shards=paths, seq=T, batch=B + 1, seed=0)
    got, want = wrong.next(), fresh.next()  # the batcher was not advanced
    assert np.array_equal(got[0], want[0]) and got[2:] == want[2:]
    for h in (t, wrong, fresh):
        h.close()


def test_evaluation_is_the_mean_loss_on_evenly_spread_sequences(mm, tmp_path):
    # trainer.rs:485-514, through midman_train_evaluate over held-out shard files
    lengths = [300, 95, 210]
    paths = shards(tmp_path, lengths, seed=4)
    t = trainer(mm)
    for x, y in [(np.arange(B * T) % 64, (np.arange(B * T) * 7) % 64)]:
        t.step(x, y)
    before = t.params().copy()
    report = t.evaluate(paths, 3)
    assert report["batches"] == 3 and report["tokens"] == 3 * B * T
    assert t.evaluate(paths, 3) == report  # the same call gives the same number
    assert np.array_equal(bits(t.params()), bits(before))  # and does not train
    # by hand: row k of the rows taken is sequence k * len / rows, mean of the batch losses in f64
    tokens = np.concatenate([ts_tokens(p) for p in paths])
    starts = np.cumsum([0] + lengths[:-1])
    windows = [(s + j * T) for s, n in zip(starts, lengths) if n > T for j in range((n - 1) // T)]
    rows = 3 * B
    oracle_model = orc.Model(CFG, seed=0)
    oracle_model.params = t.params()
    total, total_oracle = 0.0, 0.0
    for b in range(3):
        at = [windows[(b * B + r) * len(windows) // rows] for r in range(B)]
        x = np.concatenate([tokens[a:a + T] for a in at]).astype(np.int32)
        y = np.concatenate([tokens[a + 1:a + T + 1] for a in at]).astype(np.int32)
        total += float(np.float32(t.eval(x, y, B, T)))
        total_oracle += oracle_model.loss(x, y, B, T)
    assert np.float32(report["loss"]) == np.float32(total / 3)
    assert abs(report["loss"] - total_oracle / 3) <= 1e-5 * abs(total_oracle / 3)
    # more batches than the data holds is cut to what it holds
    small = tmp_path / "small.mmtokens"
    small.write_bytes(ts.to_bytes(64, 11, np.ones(5 * T + 1, np.uint32)))
    r = t.evaluate([small], 100)
    assert (r["batches"], r["tokens"]) == (5 // B, (5 // B) * B * T)
    one = tmp_path / "one.mmtokens"
    one.write_bytes(ts.to_bytes(64, 11, np.ones(T + 1, np.uint32)))  # one sequence: a batch of one row
    r = t.evaluate([one], 4)
    assert (r["batches"], r["tokens"]) == (1, T)
    t.close()


def test_evaluation_refuses_what_does_not_fit(mm, tmp_path):
    # trainer.rs:517-527
    t = trainer(mm)
    paths = shards(tmp_path, [300], seed=5)
    other_vocab = tmp_path / "v.mmtokens"
    other_vocab.write_bytes(ts.to_bytes(65, 0, np.ones(100, np.uint32)))
    empty = tmp_path / "e.mmtokens"
    empty.write_bytes(ts.to_bytes(64, 0, np.ones(T, np.uint32)))  # shorter than one window
    for args, mention in [((paths, 0), "nothing"), (([other_vocab], 2), "vocabulary"), (([empty], 2), "nothing"),
                          (([], 2), "empty")]:
        with pytest.raises(mm.MidmanError) as e:
            t.evaluate(*args)
        assert e.value.status == -1 and mention in e.value.message, (args, e.value.message)
    t.close()


def test_params_and_grads_entry_points_read_one_tensor(mm, tmp_path):
    # midman_train_params / midman_train_grads: midman_train_read with which = 0 / 1
    t = trainer(mm)
    x = (np.arange(B * T) % 64).astype(np.int32)
    t.loss_and_grads(x, x[::-1].copy())
    lib = mm.load()
    for i in (0, 3):
        assert lib.midman_train_params(t.h, i) == 0
        assert np.array_equal(mm.floats(), t.read(0, i))
        assert lib.midman_train_grads(t.h, i) == 0
        assert np.array_equal(mm.floats(), t.read(1, i))
    assert lib.midman_train_grads(t.h, 10**6) == -4  # MIDMAN_ERR_INDEX
    t.close()
