"""The C-ABI library on the CPU: it loads, exports every declared symbol, and its
stateless calls (no GPU needed) agree with the reference's answers and the oracle.
"""
import json
import re
from pathlib import Path

import numpy as np
import pytest

import oracle as orc

ROOT = Path(__file__).resolve().parent.parent
PINS = json.loads((ROOT / "tests" / "golden" / "reference_pins.json").read_text())


def declared_symbols():
    out = []
    for h in (ROOT / "include").glob("*.h"):
        for m in re.finditer(r"(?:MIDMAN_EXPORT|MM_GPU_EXPORT)[^;]*?\b((?:midman|mm_gpu|mm_tape|mm_tensor|mm_op)_\w+)\s*\(",
                             h.read_text(),
                             re.S):
            out.append(m.group(1))
    return sorted(set(out))


def test_every_declared_symbol_is_exported(mm):
    syms = declared_symbols()
    assert len(syms) >= 30
    lib = mm.load()
    for s in syms:
        assert hasattr(lib, s), s
    assert set(syms) == set(mm.GPU_SYMBOLS + mm.API_SYMBOLS + mm.TENSOR_SYMBOLS)


def test_abi_version_and_alloc(mm):
    lib = mm.load()
    assert lib.midman_abi_version() == 1
    p = lib.midman_alloc(24)
    assert p and (np.ctypeslib.as_array(p, shape=(1,)).ctypes.data % 8 == 0)
    lib.midman_free(p, 24)
    lib.midman_free(None, 0)


def test_describe_lists_presets_with_exact_counts(mm):
    d = mm.describe()
    assert d["abi"] == 1 and d["limits"] == {"max_params": 8000000, "max_tokens": 4096}
    assert [p["name"] for p in d["presets"]] == list(orc.PRESETS)
    for p in d["presets"]:
        assert p["params"] == PINS["preset_params"][p["name"]]
    assert d["config_fields"][0] == "vocab_size" and d["hyper_fields"][-1] == "beta2"


def test_preset_config_and_bad_index(mm):
    for i, name in enumerate(orc.PRESETS):
        np.testing.assert_array_equal(mm.preset_config(i), orc.preset(name).astype(np.float32).astype(np.float64))
    with pytest.raises(mm.MidmanError) as e:
        mm.preset_config(6)
    assert e.value.status == -1


def test_config_report_valid_and_invalid(mm):
    r = mm.config_report(orc.preset("smoke"))
    want = orc.param_breakdown(orc.preset("smoke"))
    assert r["valid"] and r["head_dim"] == 16 and r["kv_dim"] == 64
    assert r["params"] == want
    bad = orc.preset("smoke")
    bad[3] = 3
    r = mm.config_report(bad)
    assert r == {"valid": False, "error": r["error"]} and "n_heads" in r["error"]
    bad = orc.preset("smoke")
    bad[1] = 1.5
    with pytest.raises(mm.MidmanError) as e:
        mm.config_report(bad)
    assert e.value.status == -1 and "whole number" in e.value.message


def test_rope_table_is_bit_identical_to_the_oracle(mm):
    for hd, t in ((4, 5), (64, 128), (128, 2048)):
        c, s = mm.rope_table(hd, t, 10000.0)
        oc, os_ = orc.rope_table(hd, t, 10000.0)
        assert np.array_equal(c.view(np.uint32), oc.view(np.uint32))
        assert np.array_equal(s.view(np.uint32), os_.view(np.uint32))
    with pytest.raises(mm.MidmanError):
        mm.rope_table(3, 4, 10000.0)


def test_invalid_handles_are_argument_errors(mm):
    lib = mm.load()
    assert lib.midman_lab_step(12345, 1) == -1
    assert "not a live lab handle" in mm.error()
    assert lib.midman_train_destroy(7) == -1
    assert lib.midman_lab_destroy(0) == -1
