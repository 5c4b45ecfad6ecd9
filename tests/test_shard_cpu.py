"""Token shards and the batcher over them, without a GPU.

The library's reader (midman_shard_read / midman_shard_inspect), writer
(midman_shard_write) and SHA-256 (midman_sha256) against the reference's rules:
the cases follow the unit tests of crates/midman-data/src/shard.rs:264-457 and
the hashlib vectors of crates/midman-data/tests/reference_vectors.rs (rebuilt by
tests/golden/make_sha256_vectors.py). Files for the reader come from
oracle/token_shard.py, a restatement of TokenShard::to_bytes over hashlib. The
batcher over several shard files (midman_batcher_open, Sequences::new and
Batcher of batch.rs:38-248) is checked against the oracle's batcher.
"""
import struct
from pathlib import Path

import numpy as np
import pytest

import oracle as orc
import token_shard as ts

ERR_ARGUMENT, ERR_OTHER = -1, -5
GOLDEN = Path(__file__).resolve().parent / "golden"


def message(n):
    return bytes((31 * j + 7 * n + 5) % 256 for j in range(n))


def test_sha256_matches_the_hashlib_vectors(mm):
    lines = (GOLDEN / "sha256_vectors.txt").read_text().split("\n")
    vectors = [(int(a), b) for a, b in (line.split(" ") for line in lines if line)]
    lengths = [n for n, _ in vectors]
    assert len(vectors) == 309 and all(n in lengths for n in range(301)) and 100003 in lengths
    for n, digest in vectors:
        assert mm.sha256(message(n)).hex() == digest, n


@pytest.fixture()
def read(mm, tmp_path):
    def run(data: bytes):
        path = tmp_path / "s.mmtokens"
        path.write_bytes(data)
        return mm.shard_read(path)
    return run


def reason(mm, read, data):
    with pytest.raises(mm.MidmanError) as e:
        read(data)
    assert e.value.status == ERR_OTHER
    return e.value.message


def test_the_file_has_exactly_this_layout(mm, tmp_path, read):
    # shard.rs:291-309: vocabulary 300, end-of-text 256, ids 1 2 3 256 in two bytes each
    want_body = ("4d4d544f4b454e53" "01000000" "02000000" "2c010000" "00010000" "0400000000000000"
                 "0100020003000001")
    data = ts.to_bytes(300, 256, [1, 2, 3, 256])
    assert data[:-32].hex() == want_body and len(data) == 32 + 8 + 32
    path = tmp_path / "layout.mmtokens"
    mm.shard_write(path, 300, 256, [1, 2, 3, 256])
    assert path.read_bytes() == data
    assert mm.sha256(data[:-32]) == data[-32:]
    info, tokens = read(data)
    assert info == {"vocab_size": 300, "eos": 256, "tokens": 4, "token_width": 2}
    assert tokens.tolist() == [1, 2, 3, 256]


def test_four_byte_ids_are_used_above_65536(mm, tmp_path):
    # shard.rs:311-321
    p = tmp_path / "a.mmtokens"
    mm.shard_write(p, 65537, 0, [65536, 7])
    b = p.read_bytes()
    assert b[12:16] == struct.pack("<I", 4) and len(b) == 32 + 2 * 4 + 32 and b[32:36] == struct.pack("<I", 65536)
    mm.shard_write(p, 65536, 0, [65535, 7])
    b = p.read_bytes()
    assert b[12:16] == struct.pack("<I", 2) and len(b) == 32 + 2 * 2 + 32 and b[32:34] == struct.pack("<H", 65535)


@pytest.mark.parametrize("vocab,tokens", [(256, [0, 255, 1, 2, 3]), (65536, [0, 65535, 40000]),
                                          (65537, [0, 65536, 40000]),
                                          (4_000_000_000, [0, 3_999_999_999, 1_234_567_890]), (300, [])])
def test_round_trips_in_both_widths_and_empty(mm, tmp_path, vocab, tokens):
    # shard.rs:323-339
    p = tmp_path / "r.mmtokens"
    mm.shard_write(p, vocab, 0, np.array(tokens, np.uint64).astype(np.uint32))
    assert p.read_bytes() == ts.to_bytes(vocab, 0, tokens)
    info, back = mm.shard_read(p)
    assert back.tolist() == tokens
    assert (info["vocab_size"], info["eos"], info["tokens"]) == (vocab, 0, len(tokens))


def test_construction_checks_the_vocabulary(mm, tmp_path):
    # shard.rs:341-349
    p = tmp_path / "c.mmtokens"
    for vocab, eos, tokens, mention in [(0, 0, [], "vocabulary size is 0"), (10, 10, [], "end-of-text"),
                                        (10, 3, [1, 2, 10, 4], "token 10 at position 2")]:
        with pytest.raises(mm.MidmanError) as e:
            mm.shard_write(p, vocab, eos, tokens)
        assert e.value.status == ERR_ARGUMENT and mention in e.value.message
        assert not p.exists() and not Path(str(p) + ".tmp").exists()
    mm.shard_write(p, 10, 9, [9, 0])


def test_the_reader_refuses_a_wrong_header_each_with_its_reason(mm, read):
    # shard.rs:351-379
    good = ts.raw(1, 2, 300, 256, 2, bytes([1, 0, 2, 0]))
    assert read(good)[1].tolist() == [1, 2]
    bad = bytearray(good)
    bad[0] = ord("X")
    assert "MMTOKENS" in reason(mm, read, bytes(bad))
    for version in (2, 0):
        text = reason(mm, read, ts.raw(version, 2, 300, 256, 2, bytes([1, 0, 2, 0])))
        assert f"version {version}" in text and "1" in text
    for width in (0, 1, 3, 4, 8):
        assert "token width" in reason(mm, read, ts.raw(1, width, 300, 256, 2, bytes([1, 0, 2, 0, 0, 0, 0, 0])))
    assert "token width" in reason(mm, read, ts.raw(1, 2, 65537, 0, 1, bytes([1, 0])))
    assert "vocabulary size is 0" in reason(mm, read, ts.raw(1, 2, 0, 0, 0, b""))
    assert "end-of-text" in reason(mm, read, ts.raw(1, 2, 300, 300, 0, b""))
    assert read(ts.raw(1, 2, 300, 299, 0, b""))[0]["tokens"] == 0


def test_the_reader_refuses_a_wrong_length_for_every_cut_and_extension(mm, read):
    # shard.rs:381-400
    good = ts.to_bytes(300, 0, [1, 2, 3, 4, 5])
    for cut in range(len(good)):
        reason(mm, read, good[:cut])
    assert "do not make a file" in reason(mm, read, good + b"\0")
    assert "3 tokens" in reason(mm, read, ts.raw(1, 2, 300, 0, 3, bytes([1, 0, 2, 0])))
    for count in (2 ** 64 - 1, (2 ** 64 - 1) // 2, 1 << 62):
        assert "do not make a file" in reason(mm, read, ts.raw(1, 2, 300, 0, count, b""))


def test_the_reader_refuses_damage_anywhere_in_the_file(mm, read):
    # shard.rs:402-419: every flipped bit is an error, never a wrong shard
    good = ts.to_bytes(300, 0, [1, 2, 3, 4, 5])
    for index in range(len(good)):
        for bit in (0, 7):
            bad = bytearray(good)
            bad[index] ^= 1 << bit
            reason(mm, read, bytes(bad))
    bad = bytearray(good)
    bad[34] ^= 0x10
    assert "checksum" in reason(mm, read, bytes(bad))


def test_a_token_outside_the_vocabulary_is_refused_even_with_a_valid_checksum(mm, read):
    # shard.rs:421-427: ids 1, 300, 2
    assert "token 300 at position 1" in reason(mm, read, ts.raw(1, 2, 300, 0, 3, bytes([1, 0, 44, 1, 2, 0])))


def test_save_replaces_the_file_and_leaves_no_temporary(mm, tmp_path):
    # shard.rs:429-455
    p = tmp_path / "s.mmtokens"
    mm.shard_write(p, 300, 0, [1, 2, 3])
    mm.shard_write(p, 300, 5, [7, 8])
    assert p.read_bytes() == ts.to_bytes(300, 5, [7, 8])
    assert sorted(x.name for x in tmp_path.iterdir()) == ["s.mmtokens"]
    with pytest.raises(mm.MidmanError) as e:
        mm.shard_write(tmp_path / "no-such-dir" / "s.mmtokens", 300, 0, [1])
    assert e.value.status == ERR_OTHER
    with pytest.raises(mm.MidmanError) as e:
        mm.shard_read(tmp_path / "missing.mmtokens")
    assert e.value.status == ERR_OTHER and "missing.mmtokens" in e.value.message


def write_shards(tmp_path, lengths, vocab, seed, eos=0):
    r = np.random.default_rng(seed)
    paths, parts = [], []
    for i, n in enumerate(lengths):
        t = r.integers(0, vocab, n).astype(np.uint32)
        p = tmp_path / f"shard-{i:03d}.mmtokens"
        p.write_bytes(ts.to_bytes(vocab, eos, t))
        paths.append(p)
        parts.append(t)
    return paths, parts


def test_batches_over_shard_files_match_the_oracle(mm, tmp_path):
    # windows never cross a shard; shards shorter than a window give none (batch.rs:61-68, :96-106)
    lengths = [50, 3, 0, 17, 9, 33, 8]
    seq, batch = 8, 3
    paths, parts = write_shards(tmp_path, lengths, 70000, 1)  # four-byte ids
    ours = mm.Batcher(shards=paths, seq=seq, batch=batch, seed=11)
    ref = orc.Batcher(np.concatenate(parts), seq, batch, 11, shard_lengths=lengths)
    windows = sum((n - 1) // seq for n in lengths if n > seq)
    assert len(ref) == windows == 6 + 2 + 1 + 4
    for _ in range(3 * (windows // batch) + 1):  # a few epochs
        i, t, e, x = ours.next()
        ri, rt, re_, rx = ref.next()
        assert np.array_equal(i, ri) and np.array_equal(t, rt) and (e, x) == (re_, rx)
    ours.close()


def test_each_window_comes_from_one_shard(mm, tmp_path):
    seq = 4
    lengths = [9, 13, 5]
    parts = [np.full(n, k, np.uint32) for k, n in enumerate(lengths)]  # shard k holds only id k
    paths = []
    for k, t in enumerate(parts):
        p = tmp_path / f"{k}.mmtokens"
        mm.shard_write(p, 10, 0, t)
        paths.append(p)
    b = mm.Batcher(shards=paths, seq=seq, batch=1, seed=3)
    seen = set()
    for _ in range(2 + 3 + 1):
        i, t, _, _ = b.next()
        assert len(set(i.tolist()) | set(t.tolist())) == 1
        seen.add(int(i[0]))
    assert seen == {0, 1, 2}
    b.close()


def test_seek_gives_the_batches_of_a_continuous_run(mm, tmp_path):
    lengths = [40, 25, 61]
    seq, batch = 6, 2
    paths, parts = write_shards(tmp_path, lengths, 500, 2)
    cont = mm.Batcher(shards=paths, seq=seq, batch=batch, seed=4)
    run = [cont.next() for _ in range(25)]
    per_epoch = (6 + 4 + 10) // batch
    for k in (0, 3, 9, 10, 17):
        b = mm.Batcher(shards=paths, seq=seq, batch=batch, seed=4)
        place = b.seek(k // per_epoch, k % per_epoch)
        assert place["epoch"] == k // per_epoch and place["position"] == k % per_epoch
        for want in run[k:k + 4]:
            got = b.next()
            assert np.array_equal(got[0], want[0]) and np.array_equal(got[1], want[1]) and got[2:] == want[2:]
        b.close()
    with pytest.raises(mm.MidmanError) as e:
        cont.seek(0, per_epoch + 1)
    assert e.value.status == ERR_ARGUMENT
    cont.close()


def test_opening_shards_checks_them(mm, tmp_path):
    a = tmp_path / "a.mmtokens"
    b = tmp_path / "b.mmtokens"
    c = tmp_path / "c.mmtokens"
    a.write_bytes(ts.to_bytes(300, 0, np.arange(100) % 300))
    b.write_bytes(ts.to_bytes(301, 0, np.arange(100) % 300))
    c.write_bytes(ts.to_bytes(300, 1, np.arange(100) % 300))
    for other in (b, c):  # batch.rs:45-58
        with pytest.raises(mm.MidmanError) as e:
            mm.Batcher(shards=[a, other], seq=8, batch=2)
        assert e.value.status == ERR_ARGUMENT and "shard 1 has vocabulary size" in e.value.message
    damaged = bytearray(a.read_bytes())
    damaged[40] ^= 1
    d = tmp_path / "d.mmtokens"
    d.write_bytes(bytes(damaged))
    with pytest.raises(mm.MidmanError) as e:
        mm.Batcher(shards=[a, d], seq=8, batch=2)
    assert e.value.status == ERR_OTHER and "checksum" in e.value.message
    with pytest.raises(mm.MidmanError) as e:
        mm.Batcher(shards=[a, tmp_path / "none.mmtokens"], seq=8, batch=2)
    assert e.value.status == ERR_OTHER
    with pytest.raises(mm.MidmanError) as e:
        mm.Batcher(shards=[], seq=8, batch=2)
    assert e.value.status == ERR_ARGUMENT
    with pytest.raises(mm.MidmanError):  # fewer windows than one batch
        mm.Batcher(shards=[a], seq=60, batch=2)
    ok = mm.Batcher(shards=[a, a], seq=8, batch=2)
    assert ok.seek(0, 0)["sequences"] == 2 * 12
    ok.close()
