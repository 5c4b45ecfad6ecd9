"""Writes sha256_vectors.txt: `length digest` lines made with Python's hashlib.

The messages follow crates/midman-data/tests/reference_vectors.rs:5-15 (and the
fixture generator it names): byte j of the message of length n is
(31 * j + 7 * n + 5) mod 256. The lengths are every length up to 300 and the
block-boundary and large lengths of the reference fixture (reference_vectors.rs:
28-33 pins 309 lines, 0..=300 and 100,003 among them).

    python tests/golden/make_sha256_vectors.py
"""
import hashlib
from pathlib import Path

LENGTHS = list(range(301)) + [511, 512, 513, 1000, 4096, 65535, 65536, 100003]


def message(n: int) -> bytes:
    return bytes((31 * j + 7 * n + 5) % 256 for j in range(n))


def main() -> None:
    lines = [f"{n} {hashlib.sha256(message(n)).hexdigest()}" for n in LENGTHS]
    (Path(__file__).resolve().parent / "sha256_vectors.txt").write_text("\n".join(lines) + "\n")


if __name__ == "__main__":
    main()
