"""The reference's own C ABI smoke tests run against this library.

crates/midman-api/ffi-smoke-test/test.c (a C11 caller: version and layout, buffers
from midman_alloc, malformed arguments, lab lifecycle, slots, invented handles,
refused creations, blow-up to MIDMAN_STOPPED, replaced results, seeds, RoPE tables)
and cxx_check.cpp (the header from C++17), compiled unchanged by `make -C oracle ffi`
where the reference checkout is present: test.c once against the reference's own
midman_api.h (a caller built for the reference) and once against include/midman_api.h.
Each binary prints "ok:"/"FAIL:" lines and "=== N check(s) failed ===". The labs
need the GPU, so these run with the GPU tests; they are skipped where the binaries
were not built.
"""
import subprocess
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

REF = Path(__file__).resolve().parent.parent / "oracle" / "_ref"


@pytest.mark.parametrize("binary", ["ffi_test_c_refheader", "ffi_test_c", "ffi_cxx_check"])
def test_reference_ffi_smoke_test_passes(mm, binary):
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    exe = REF / binary
    if not exe.exists():
        pytest.skip(f"{binary} not built (make -C oracle ffi needs the reference checkout)")
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=600)
    fails = [line for line in r.stdout.splitlines() if line.startswith("FAIL")]
    assert r.returncode == 0 and not fails, (fails, r.stdout[-3000:], r.stderr[-2000:])
    assert "=== 0 check(s) failed ===" in r.stdout
    assert sum(line.startswith("ok:") for line in r.stdout.splitlines()) >= (40 if "test_c" in binary else 6)
