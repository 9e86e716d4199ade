"""VAE tensors from a safetensors file (the reference's bundle loader for
`vae.safetensors`, src/artifact.rs:585-760, without the manifest and SHA-256
policy of the full bundle).

The file is read with bounded sizes and validated the way the reference
validates it before any tensor is built: an 8-byte little-endian header
length, a JSON header whose tensors cover the data region exactly once in
offset order, plain diffusers names (ASCII letters, digits, '.', '_', '-';
no empty dotted parts; no 'unet.', 'module.', '_orig_mod.' prefixes or LoRA
parts), dtypes F16 / BF16 / F32, ranks 1..8, dimensions 1..1e6 and per-tensor
and aggregate byte limits. Tensors are returned as float32 numpy arrays keyed
by name, ready for ``NativeModel`` (which repacks them once into the device
layout).
"""
from __future__ import annotations

import json
import os
import re
import struct
from dataclasses import dataclass
from typing import Dict

import numpy as np

from ._lib import InvalidArtifact


@dataclass
class ArtifactLimits:
    """src/artifact.rs:110-145 defaults."""
    max_file_bytes: int = 24 * 1024 ** 3
    max_header_bytes: int = 16 * 1024 ** 2
    max_tensors: int = 30_000
    max_tensor_bytes: int = 1024 ** 3
    max_total_tensor_bytes: int = 32 * 1024 ** 3
    max_rank: int = 8
    max_dimension: int = 1_000_000
    max_name_bytes: int = 512


_DTYPES = {"F32": (np.float32, 4), "F16": (np.float16, 2), "BF16": (np.uint16, 2)}
_NAME = re.compile(r"^[A-Za-z0-9._-]+$")
_FOREIGN = ("unet.", "module.", "_orig_mod.")


def _name_ok(name: str, limits: ArtifactLimits) -> bool:
    return (0 < len(name.encode()) <= limits.max_name_bytes and _NAME.match(name) is not None
            and all(name.split(".")))


def read_safetensors(path: str, limits: ArtifactLimits = None) -> Dict[str, np.ndarray]:
    """Tensors of one safetensors file as float32 arrays (artifact.rs:671-760)."""
    limits = limits or ArtifactLimits()
    if not os.path.isfile(path):
        raise InvalidArtifact(f"{path} is not a regular file")
    size = os.path.getsize(path)
    if size < 8 or size > limits.max_file_bytes:
        raise InvalidArtifact(f"{path} has an invalid or oversized file length")
    with open(path, "rb") as f:
        (header_len,) = struct.unpack("<Q", f.read(8))
        if header_len == 0 or header_len > limits.max_header_bytes or header_len + 8 > size:
            raise InvalidArtifact("invalid or oversized safetensors header")
        try:
            header = json.loads(f.read(header_len))
        except (ValueError, UnicodeDecodeError) as e:
            raise InvalidArtifact(f"invalid safetensors header: {e}") from None
        if not isinstance(header, dict):
            raise InvalidArtifact("invalid safetensors header")
        header.pop("__metadata__", None)
        if not header or len(header) > limits.max_tensors:
            raise InvalidArtifact("invalid or excessive safetensors tensor count")
        entries = []
        for name, info in header.items():
            try:
                dtype, shape, (begin, end) = info["dtype"], list(info["shape"]), info["data_offsets"]
            except (KeyError, TypeError, ValueError):
                raise InvalidArtifact(f"invalid safetensors entry {name!r}") from None
            entries.append((int(begin), int(end), name, dtype, shape))
        entries.sort()
        offset, decoded = 0, 0
        for begin, end, name, dtype, shape in entries:
            if begin != offset:
                raise InvalidArtifact("safetensors data offsets overlap or contain gaps")
            if not _name_ok(name, limits):
                raise InvalidArtifact(f"invalid tensor name {name!r}")
            if dtype not in _DTYPES:
                raise InvalidArtifact(f"{name} has an unsupported dtype")
            if (not shape or len(shape) > limits.max_rank
                    or any(not isinstance(d, int) or d <= 0 or d > limits.max_dimension
                           for d in shape)):
                raise InvalidArtifact(f"{name} has an invalid or oversized shape")
            count = int(np.prod(shape, dtype=np.int64))
            source = count * _DTYPES[dtype][1]
            if source > limits.max_tensor_bytes or count * 4 > limits.max_tensor_bytes \
                    or end - begin != source:
                raise InvalidArtifact(f"{name} has invalid offsets or exceeds the tensor limit")
            decoded += count * 4
            offset = end
        if offset + header_len + 8 != size:
            raise InvalidArtifact("safetensors offsets do not cover the file")
        if decoded > limits.max_total_tensor_bytes:
            raise InvalidArtifact("aggregate tensor budget exceeded")
        out: Dict[str, np.ndarray] = {}
        for begin, end, name, dtype, shape in entries:
            raw = f.read(end - begin)
            if len(raw) != end - begin:
                raise InvalidArtifact(f"{path} is truncated")
            np_type = _DTYPES[dtype][0]
            a = np.frombuffer(raw, dtype=np.dtype(np_type).newbyteorder("<")).reshape(shape)
            if dtype == "BF16":
                a = (a.astype(np.uint32) << 16).view(np.float32)
            out[name] = np.ascontiguousarray(a, dtype=np.float32)
    if any(n.startswith(_FOREIGN) or ".base_layer." in n or ".lora_" in n for n in out):
        raise InvalidArtifact("vae tensor names must be plain diffusers names")
    return out


def write_safetensors(path: str, tensors: Dict[str, np.ndarray], dtype: str = "F32") -> None:
    """Write float tensors (F32, F16 or BF16 storage, round to nearest even)."""
    if dtype not in _DTYPES:
        raise InvalidArtifact("safetensors dtype must be F32, F16 or BF16")
    header, blobs, offset = {}, [], 0
    for name in sorted(tensors):
        a = np.ascontiguousarray(tensors[name], np.float32)
        if dtype == "F32":
            data = a.astype("<f4").tobytes()
        elif dtype == "F16":
            data = a.astype("<f2").tobytes()
        else:
            bits = a.view(np.uint32).astype(np.uint64)
            bits = (bits + 0x7FFF + ((bits >> 16) & 1)) >> 16  # round to nearest even
            data = bits.astype("<u2").tobytes()
        header[name] = {"dtype": dtype, "shape": list(a.shape),
                        "data_offsets": [offset, offset + len(data)]}
        blobs.append(data)
        offset += len(data)
    head = json.dumps(header, separators=(",", ":")).encode()
    head += b" " * (-len(head) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(head)))
        f.write(head)
        for b in blobs:
            f.write(b)
