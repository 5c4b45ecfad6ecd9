"""Test infrastructure: a Python restatement of the reference's token-shard writer.

It makes `.mmtokens` files for the tests of the library's shard reader and input
pipeline (midman_shard_read, midman_batcher_open, midman_train_run); nothing in
the library uses it. The digest comes from Python's hashlib, independent of the
library's own SHA-256.

* TokenShard::to_bytes (crates/midman-data/src/shard.rs:113-135): the magic
  `MMTOKENS`, then version, token width, vocabulary size and end-of-text id as
  little-endian u32, the token count as little-endian u64, the ids as
  little-endian u16 (vocabularies of up to 65,536 ids, shard.rs:28-34) or u32,
  and the SHA-256 of all bytes before it.
* `raw` is the reference test helper `file` (shard.rs:273-285): any header
  fields and payload, with a correct checksum.
"""
from __future__ import annotations

import hashlib
import struct

import numpy as np

MAGIC = b"MMTOKENS"
VERSION = 1


def width_for(vocab_size: int) -> int:
    return 2 if vocab_size <= 65536 else 4


def raw(version: int, width: int, vocab: int, eos: int, count: int, payload: bytes) -> bytes:
    body = MAGIC + struct.pack("<IIIIQ", version, width, vocab, eos, count) + bytes(payload)
    return body + hashlib.sha256(body).digest()


def to_bytes(vocab_size: int, eos: int, tokens) -> bytes:
    t = np.asarray(tokens, np.uint64)
    assert vocab_size > 0 and eos < vocab_size and (t.size == 0 or int(t.max()) < vocab_size)
    w = width_for(vocab_size)
    payload = t.astype("<u2" if w == 2 else "<u4").tobytes()
    return raw(VERSION, w, vocab_size, eos, t.size, payload)
