"""Checks that every known answer in reference_pins.json appears in the reference file it cites.

Run where the reference tree is checked out (its directory as the argument, or in
MIDMAN_REFERENCE_DIR):
    python tests/golden/check_provenance.py [REFERENCE_DIR]
Numbers are compared by their digits (underscores removed, hex lower-cased), so a value
pinned from `0x99ec_5f36_cb75_f2b4` or `0.602_082_3` is found.
"""
import json
import os
import re
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent


def numbers(text):
    """Every numeric literal of the file: hex strings, and all others as floats."""
    text = text.replace("_", "").lower()
    hexes = set(re.findall(r"0x[0-9a-f]+", text))
    vals = set()
    for lit in re.findall(r"(?<![0-9a-fx.])\d+(?:\.\d*)?(?:e-?\d+)?", text):
        try:
            vals.add(float(lit))
        except ValueError:
            pass
    return hexes, vals


def flatten(v):
    if isinstance(v, (list, tuple)):
        for x in v:
            yield from flatten(x)
    elif isinstance(v, (int, float)) and not isinstance(v, bool):
        yield v
    elif isinstance(v, str) and v.startswith("0x"):
        yield v


def present(v, found):
    hexes, vals = found
    if isinstance(v, str):
        return v.lower() in hexes
    a = abs(float(v))
    return any(abs(a - x) <= 1e-12 * max(1.0, a) for x in vals)


def main(ref_dir):
    pins = json.loads((HERE / "reference_pins.json").read_text())
    missing = 0
    for key, entry in pins.items():
        if key.startswith("_") or "cite" not in entry:
            continue
        path = Path(ref_dir) / entry["cite"].split(":")[0]
        found = numbers(path.read_text())
        for field, value in entry.items():
            if field in ("cite", "tol", "derived") or field.endswith("_formula") or field in entry.get("derived", {}):
                continue
            for v in flatten(value):
                if not present(v, found):
                    missing += 1
                    print(f"{key}.{field}: {v!r} not found in {entry['cite']}")
    print("all pinned literals found" if not missing else f"{missing} literals not found")
    return 1 if missing else 0


if __name__ == "__main__":
    default = os.environ.get("MIDMAN_REFERENCE_DIR", str(Path(__file__).resolve().parents[3] / "reference"))
    sys.exit(main(sys.argv[1] if len(sys.argv) > 1 else default))
