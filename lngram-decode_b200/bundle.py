"""Drafter bundles: the reference's flat ``MRBDRFT1`` file format, read and written here.

Format (the interface of ``drafting/export_drafter.py:12-35``; every number little-endian):

    bytes [0, 8)        the magic ``MRBDRFT1``
    bytes [8, 16)       u64 H, the byte length of the JSON header
    bytes [16, 16 + H)  the header: UTF-8 JSON with sorted keys,
                        ``{"arrays": {name: {dtype, nbytes, offset, shape}}, "config", "source", "version": 1}``
    then each array's raw C-order bytes at its ``offset``, a multiple of 64; zero bytes fill the gaps.

Placement rule (needed for byte-identical files): the first array starts at the first multiple of 64
at or after 16 + H + 256, and each next array at the first multiple of 64 after the previous one
ends, in the dictionary's order.  Because the offsets are part of the header, H and the offsets are
solved together: start from the header with every offset 0 and re-place until the header length no
longer changes (the same fixed point the reference's writer reaches from the same start).
"""

from __future__ import annotations

import json
import struct
from dataclasses import dataclass
from pathlib import Path

import numpy as np

MAGIC = b"MRBDRFT1"
VERSION = 1
ALIGN = 64
PREFIX = len(MAGIC) + 8     # magic + header length
HEADER_SLACK = 256          # spare bytes between the header and the first array


@dataclass
class Bundle:
    config: dict
    arrays: dict   # name -> numpy array (memory-mapped when loaded with mmap=True)
    source: dict


def _round_up(n: int) -> int:
    return -(-n // ALIGN) * ALIGN


def _header_bytes(config: dict, meta: dict, source: dict) -> bytes:
    doc = {"version": VERSION, "config": config, "arrays": meta, "source": source}
    return json.dumps(doc, sort_keys=True).encode("utf-8")


def _offsets(header_len: int, sizes: list) -> list:
    """Array offsets for a header of ``header_len`` bytes and arrays of ``sizes`` bytes."""
    out, pos = [], _round_up(PREFIX + header_len + HEADER_SLACK)
    for n in sizes:
        out.append(pos)
        pos = _round_up(pos + n)
    return out


def _layout(config: dict, arrays: dict, source: dict) -> tuple[bytes, dict]:
    """(header bytes, per-array metadata) at the fixed point of header length and offsets."""
    names = list(arrays)
    sizes = [int(arrays[k].nbytes) for k in names]

    def meta_for(offs):
        return {k: {"dtype": arrays[k].dtype.str, "shape": [int(s) for s in arrays[k].shape], "offset": int(o),
                    "nbytes": n} for k, o, n in zip(names, offs, sizes)}

    header = _header_bytes(config, meta_for([0] * len(names)), source)
    for _ in range(64):
        meta = meta_for(_offsets(len(header), sizes))
        placed = _header_bytes(config, meta, source)
        if len(placed) == len(header):
            return placed, meta
        header = placed
    raise RuntimeError("bundle header layout did not converge")


def write_bundle(path: str | Path, config: dict, arrays: dict, source: dict | None = None) -> Path:
    """Write ``arrays`` (name -> numpy array, in this order) and the JSON ``config`` / ``source``."""
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    arrays = {k: np.ascontiguousarray(v) for k, v in arrays.items()}
    header, meta = _layout(config, arrays, source or {})
    with open(path, "wb") as f:
        f.write(MAGIC + struct.pack("<Q", len(header)) + header)
        for name, a in arrays.items():
            gap = meta[name]["offset"] - f.tell()
            if gap:
                f.write(bytes(gap))
            little = a.astype(a.dtype.newbyteorder("<"), copy=False) if a.dtype.byteorder == ">" else a
            f.write(memoryview(little).cast("B"))
    return path


def read_header(path: str | Path) -> dict:
    """The decoded JSON header; ValueError when the file does not start with the magic."""
    with open(path, "rb") as f:
        prefix = f.read(PREFIX)
        if len(prefix) < PREFIX or prefix[:len(MAGIC)] != MAGIC:
            raise ValueError(f"{path}: missing the {MAGIC.decode()} magic, not a drafter bundle")
        (hlen,) = struct.unpack("<Q", prefix[len(MAGIC):])
        return json.loads(f.read(hlen))


def load_bundle(path: str | Path, mmap: bool = True) -> Bundle:
    """Every array of the bundle: read-only memory maps (``mmap``) or in-memory copies."""
    head = read_header(path)
    if head.get("version") != VERSION:
        raise ValueError(f"{path}: bundle format version {head.get('version')}, this reader handles {VERSION}")
    arrays = {}
    for name, m in head["arrays"].items():
        dt, shape = np.dtype(m["dtype"]), tuple(m["shape"])
        count = int(np.prod(shape, dtype=np.int64))
        if mmap and m["nbytes"]:
            arrays[name] = np.memmap(path, dtype=dt, mode="r", offset=m["offset"], shape=shape)
        else:
            arrays[name] = np.fromfile(path, dtype=dt, count=count, offset=m["offset"]).reshape(shape)
    return Bundle(head["config"], arrays, head.get("source", {}))


def as_bundle(bundle) -> Bundle:
    """A Bundle from a Bundle, a path, or any object with ``config`` and ``arrays`` (the reference's
    own ``drafting.export_drafter.Bundle`` included)."""
    if isinstance(bundle, (str, Path)):
        return load_bundle(bundle)
    if isinstance(bundle, Bundle):
        return bundle
    return Bundle(dict(bundle.config), dict(bundle.arrays), dict(getattr(bundle, "source", {}) or {}))
