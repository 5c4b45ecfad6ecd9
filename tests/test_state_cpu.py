"""The state-file reader (midman_state_inspect, no GPU) against the reference's rules.

midman_state_inspect runs TensorFile::from_bytes (crates/midman-checkpoint/src/
safetensors.rs:270-353, with the header reader of json.rs) and, for a file whose
`format` entry names a training state, progress_of (crates/midman-training/src/
state.rs:125-173). The
cases follow the reference's own tests (safetensors.rs:447-700, state.rs:507-540);
the files are written with oracle/safetensors.py, whose output is pinned here to
the header the reference's writer test spells out (safetensors.rs:513-526).
"""
import struct

import numpy as np
import pytest

import safetensors as st

ERR_ARGUMENT, ERR_OTHER = -1, -5


@pytest.fixture()
def inspect(mm, tmp_path):
    def run(data: bytes):
        path = tmp_path / "f.safetensors"
        path.write_bytes(data)
        return mm.state_inspect(path)
    return run


def floats(*xs):
    return np.array(xs, "<f4").tobytes()


def one_tensor_header(dtype, shape, begin, end):
    return '{"a":{"dtype":"%s","shape":%s,"data_offsets":[%d,%d]}}' % (dtype, shape, begin, end)


def sample():
    return [("w", (2, 3), np.array([1.5, -2.0, 0.0, 3.25, 1e-30, 1e30], np.float32)),
            ("b", (3,), np.array([0.1, 0.2, 0.3], np.float32))]


def test_the_python_writer_matches_the_reference_header():
    # safetensors.rs:513-526: sorted by name, metadata first, padded to 8 bytes
    b = st.to_bytes(sample(), {"format": "test"})
    n = struct.unpack("<Q", b[:8])[0]
    assert n % 8 == 0 and len(b) == 8 + n + 36
    assert b[8:8 + n].decode().rstrip() == (
        '{"__metadata__":{"format":"test"},'
        '"b":{"dtype":"F32","shape":[3],"data_offsets":[0,12]},'
        '"w":{"dtype":"F32","shape":[2,3],"data_offsets":[12,36]}}')
    assert st.to_bytes([], {}) == st.raw_file("{}      ")  # safetensors.rs:544-550


def test_a_written_file_reads_back(inspect):
    out = inspect(st.to_bytes(sample() + [("scalar", (), np.array([7.0], np.float32)),
                                          ("empty", (0,), np.zeros(0, np.float32)),
                                          ("blocks.0.attn.wq é日本", (1, 1, 2), np.array([1, 2], np.float32))],
                              {"format": "test", "note": 'quote " backslash \\ newline \n é'}))
    assert out["metadata"]["note"] == 'quote " backslash \\ newline \n é'
    names = [t["name"] for t in out["tensors"]]
    assert set(names) == {"w", "b", "scalar", "empty", "blocks.0.attn.wq é日本"}
    shapes = {t["name"]: t["shape"] for t in out["tensors"]}
    assert shapes["scalar"] == [] and shapes["empty"] == [0] and shapes["w"] == [2, 3]


def test_tensors_are_ordered_by_their_place_in_the_data(inspect):
    # safetensors.rs:552-560
    header = ('{"a":{"dtype":"F32","shape":[1],"data_offsets":[4,8]},'
              '"z":{"dtype":"F32","shape":[1],"data_offsets":[0,4]}}')
    out = inspect(st.raw_file(header, floats(1.0, 2.0)))
    assert [t["name"] for t in out["tensors"]] == ["z", "a"]
    out = inspect(st.raw_file(one_tensor_header("F32", "[1]", 0, 4) + " \n\t  ", floats(9.0)))
    assert out["tensors"][0]["data_offsets"] == [0, 4]


MALFORMED = [  # safetensors.rs:584-656, by name
    ("short prefix", bytes([2, 0, 0, 0, 0, 0, 0])),
    ("header length of u64::MAX", struct.pack("<Q", 2 ** 64 - 1) + b"{}"),
    ("header past the end of the file", struct.pack("<Q", 50) + b"{}"),
    ("header over the format limit", struct.pack("<Q", 100_000_001) + b"{}"),
    ("header not starting with {", st.raw_file(" {}")),
    ("header not UTF-8", struct.pack("<Q", 3) + bytes([ord("{"), 0xFF, ord("}")])),
    ("header not an object", st.raw_file("[]")),
    ("unsupported dtype", st.raw_file(one_tensor_header("F16", "[1]", 0, 2), b"\0\0")),
    ("lowercase dtype", st.raw_file(one_tensor_header("f32", "[1]", 0, 4), floats(1.0))),
    ("shape against range", st.raw_file(one_tensor_header("F32", "[2]", 0, 4), floats(1.0))),
    ("end before begin", st.raw_file(one_tensor_header("F32", "[1]", 4, 0), floats(1.0))),
    ("range past the data", st.raw_file(one_tensor_header("F32", "[1]", 0, 4), b"\0\0")),
    ("trailing bytes", st.raw_file(one_tensor_header("F32", "[1]", 0, 4), floats(1.0, 2.0))),
    ("gap before the first tensor", st.raw_file(one_tensor_header("F32", "[1]", 4, 8), floats(1.0, 2.0))),
    ("shape overflow", st.raw_file(one_tensor_header("F32", "[4294967296,4294967296,4294967296]", 0, 4),
                                   floats(1.0))),
    ("dimension too large for a u64", st.raw_file(one_tensor_header("F32", "[18446744073709551616]", 0, 4),
                                                  floats(1.0))),
    ("negative dimension", st.raw_file(one_tensor_header("F32", "[-1]", 0, 4), floats(1.0))),
    ("unknown field", st.raw_file('{"a":{"dtype":"F32","shape":[1],"data_offsets":[0,4],"extra":1}}', floats(1.0))),
    ("missing field", st.raw_file('{"a":{"dtype":"F32","shape":[1]}}', floats(1.0))),
    ("entry not an object", st.raw_file('{"a":1}', floats(1.0))),
    ("three offsets", st.raw_file('{"a":{"dtype":"F32","shape":[1],"data_offsets":[0,4,8]}}', floats(1.0))),
    ("metadata not strings", st.raw_file('{"__metadata__":{"k":1}}')),
    ("metadata not an object", st.raw_file('{"__metadata__":["k"]}')),
    ("duplicate tensor names", st.raw_file('{"a":{"dtype":"F32","shape":[1],"data_offsets":[0,4]},'
                                           '"a":{"dtype":"F32","shape":[1],"data_offsets":[4,8]}}',
                                           floats(1.0, 2.0))),
    # json.rs rules (json.rs:5-9, :98-280)
    ("fraction", st.raw_file(one_tensor_header("F32", "[1.0]", 0, 4), floats(1.0))),
    ("leading zero", st.raw_file(one_tensor_header("F32", "[01]", 0, 4), floats(1.0))),
    ("boolean", st.raw_file('{"__metadata__":{"k":true}}')),
    ("nesting too deep", st.raw_file('{"__metadata__":' + "[" * 9 + "]" * 9 + "}")),
    ("unpaired surrogate", st.raw_file('{"__metadata__":{"k":"\\ud800"}}')),
    ("control character", st.raw_file('{"__metadata__":{"k":"a\tb"}}')),
    ("unknown escape", st.raw_file('{"__metadata__":{"k":"\\q"}}')),
]


@pytest.mark.parametrize("case", MALFORMED, ids=[c[0] for c in MALFORMED])
def test_malformed_files_are_refused(mm, inspect, case):
    _, data = case
    with pytest.raises(mm.MidmanError) as e:
        inspect(data)
    assert e.value.status == ERR_OTHER
    assert "safetensors" in e.value.message


def test_refusals_name_what_they_refuse(mm, inspect):
    with pytest.raises(mm.MidmanError, match="limit"):
        inspect(struct.pack("<Q", 100_000_001) + b"{}")
    with pytest.raises(mm.MidmanError) as e:  # right at the limit it is the missing bytes
        inspect(struct.pack("<Q", 100_000_000) + b"{}")
    assert "limit" not in e.value.message
    with pytest.raises(mm.MidmanError, match="no gap or overlap"):  # safetensors.rs:672-677
        inspect(st.raw_file('{"a":{"dtype":"F32","shape":[2],"data_offsets":[0,8]},'
                            '"b":{"dtype":"F32","shape":[2],"data_offsets":[4,12]}}', floats(1, 2, 3)))
    with pytest.raises(mm.MidmanError, match="cover"):  # safetensors.rs:679-686
        inspect(st.raw_file(one_tensor_header("F32", "[1000000000]", 0, 4_000_000_000), floats(1.0)))
    with pytest.raises(mm.MidmanError) as e:  # safetensors.rs:688-697
        inspect(st.raw_file(one_tensor_header("BF16", "[1]", 0, 2), b"\0\0"))
    assert "`a`" in e.value.message and "BF16" in e.value.message


def state_file(**over):
    md = st.settings_metadata(8, 16, 0, 1e-3, 1e-4, 5, 100, 0.9, 0.95, 1e-8, 0.1, 1.0)
    md.update({"format": "midman-training-state", "state_version": "1", "step": "1", "epoch": "2",
               "position": "7"})
    md.update(over)
    return st.to_bytes([("param/w", (2,), np.array([1, 2], np.float32))], md)


def test_the_progress_of_a_state_file(mm, inspect):
    out = inspect(state_file())
    assert out["progress"] == {"step": 1, "epoch": 2, "position": 7}
    assert out["metadata"]["train.eps"] == "0.00000001" and out["metadata"]["train.clip_norm"] == "1"
    assert inspect(state_file(step="+3"))["progress"]["step"] == 3  # u64::from_str takes one `+`
    assert "progress" not in inspect(state_file(format="something-else"))  # not a training state
    for over, mention in [({"step": "many"}, "many"),
                          ({"position": "-3"}, "position"), ({"state_version": "9"}, "9"),
                          ({"epoch": ""}, "epoch")]:
        with pytest.raises(mm.MidmanError, match=mention) as e:
            inspect(state_file(**over))
        assert e.value.status == ERR_OTHER
    md_without_format = st.to_bytes([], {"step": "1"})
    assert "progress" not in inspect(md_without_format)  # not a state file: container only


def test_a_missing_file_is_an_error_not_a_crash(mm, tmp_path):
    with pytest.raises(mm.MidmanError):
        mm.state_inspect(tmp_path / "nope.safetensors")
    with pytest.raises(mm.MidmanError) as e:
        mm.state_inspect("")
    assert e.value.status == ERR_ARGUMENT
