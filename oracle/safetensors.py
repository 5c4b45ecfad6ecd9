"""Test infrastructure: a Python restatement of the reference's state-file writer.

It is the checker for the library's state files (midman_train_save) and a source
of hand-made files for its reader; nothing in the library uses it.

* TensorFile::write_to (crates/midman-checkpoint/src/safetensors.rs:139-222): an
  8-byte little-endian header length, a JSON header with the `__metadata__`
  object first (keys sorted), then the tensors sorted by name with consecutive
  `[begin, end)` byte ranges, the header padded with spaces to a multiple of 8,
  then the little-endian f32 data in the same order.
* json::write_string (crates/midman-checkpoint/src/json.rs:51-70): serde_json's
  escapes.
* state_to_file (crates/midman-training/src/state.rs:45-116) and
  TrainConfig::entries (crates/midman-training/src/config.rs:113-131): tensor
  names `param/<name>`, `adamw.m/<name>`, `adamw.v/<name>` and the metadata keys.
"""
from __future__ import annotations

import struct

import numpy as np


def json_string(text: str) -> str:
    out = ['"']
    for ch in text:
        c = ord(ch)
        if ch == '"':
            out.append('\\"')
        elif ch == "\\":
            out.append("\\\\")
        elif c == 0x08:
            out.append("\\b")
        elif c == 0x0C:
            out.append("\\f")
        elif ch == "\n":
            out.append("\\n")
        elif ch == "\r":
            out.append("\\r")
        elif ch == "\t":
            out.append("\\t")
        elif c < 0x20:
            out.append("\\u%04x" % c)
        else:
            out.append(ch)
    out.append('"')
    return "".join(out)


def to_bytes(tensors: list[tuple[str, tuple[int, ...], np.ndarray]], metadata: dict[str, str]) -> bytes:
    """TensorFile::to_bytes of these (name, shape, f32 values) tensors and this metadata."""
    parts = ["{"]
    first = True
    if metadata:
        parts.append('"__metadata__":{')
        parts.append(",".join(json_string(k) + ":" + json_string(v) for k, v in sorted(metadata.items(),
                                                                                     key=lambda kv: kv[0].encode())))
        parts.append("}")
        first = False
    begin = 0
    data = []
    for name, shape, values in sorted(tensors, key=lambda t: t[0].encode()):
        v = np.ascontiguousarray(values, dtype="<f4").reshape(-1)
        end = begin + 4 * v.size
        if not first:
            parts.append(",")
        first = False
        parts.append(json_string(name) + ':{"dtype":"F32","shape":[' + ",".join(str(d) for d in shape) +
                     '],"data_offsets":[' + f"{begin},{end}" + "]}")
        data.append(v.tobytes())
        begin = end
    parts.append("}")
    header = "".join(parts).encode()
    header += b" " * ((8 - len(header) % 8) % 8)
    return struct.pack("<Q", len(header)) + header + b"".join(data)


def raw_file(header: str | bytes, data: bytes = b"") -> bytes:
    """A file from a hand-written header and raw data (the reference tests' raw_file)."""
    h = header.encode() if isinstance(header, str) else header
    return struct.pack("<Q", len(h)) + h + data


def rust_f32(x: float) -> str:
    """Rust's Display of an f32: shortest round-trip digits, never an exponent."""
    return np.format_float_positional(np.float32(x), unique=True, trim="-")


def settings_metadata(batch_size, seq_len, seed, max_lr, min_lr, warmup_steps, total_steps, beta1, beta2, eps,
                      weight_decay, clip_norm) -> dict[str, str]:
    return {
        "train.batch_size": str(batch_size), "train.seq_len": str(seq_len), "train.seed": str(seed),
        "train.max_lr": rust_f32(max_lr), "train.min_lr": rust_f32(min_lr),
        "train.warmup_steps": str(warmup_steps), "train.total_steps": str(total_steps),
        "train.beta1": rust_f32(beta1), "train.beta2": rust_f32(beta2), "train.eps": rust_f32(eps),
        "train.weight_decay": rust_f32(weight_decay), "train.clip_norm": rust_f32(clip_norm),
    }


def state_bytes(params: list[tuple[str, tuple[int, ...], np.ndarray]], moments, step: int, epoch: int,
                position: int, settings: dict[str, str]) -> bytes:
    """state_to_file(...).to_bytes(): moments is a list of (name, m, v) or None before the first step."""
    md = dict(settings)
    md.update({"format": "midman-training-state", "state_version": "1", "step": str(step), "epoch": str(epoch),
               "position": str(position)})
    tensors = [("param/" + n, s, v) for n, s, v in params]
    shapes = {n: s for n, s, _ in params}
    for name, m, v in moments or []:
        tensors.append(("adamw.m/" + name, shapes[name], m))
        tensors.append(("adamw.v/" + name, shapes[name], v))
    return to_bytes(tensors, md)
