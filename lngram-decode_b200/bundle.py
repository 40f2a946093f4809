"""Drafter bundles in the reference's flat binary format (read and write).

Layout (``drafting/export_drafter.py:12-35``, all little-endian): 8-byte magic ``MRBDRFT1``,
uint64 header length H, H bytes of JSON header ``{version, config, arrays, source}``, then every
array at a 64-byte aligned absolute offset (``arrays[name] = {dtype, shape, offset, nbytes}``).
The format is kept identical so bundles exported by the reference load here unchanged.
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


@dataclass
class Bundle:
    config: dict
    arrays: dict   # name -> numpy array (memory-mapped when loaded with mmap=True)
    source: dict


def _align(x: int) -> int:
    return (x + ALIGN - 1) // ALIGN * ALIGN


def read_header(path: str | Path) -> dict:
    with open(path, "rb") as f:
        if f.read(8) != MAGIC:
            raise ValueError(f"{path}: not a drafter bundle")
        (n,) = struct.unpack("<Q", f.read(8))
        return json.loads(f.read(n).decode("utf-8"))


def load_bundle(path: str | Path, mmap: bool = True) -> Bundle:
    head = read_header(path)
    if head["version"] != VERSION:
        raise ValueError(f"bundle version {head['version']} != {VERSION}")
    arrays = {}
    for name, meta in head["arrays"].items():
        dt, shape = np.dtype(meta["dtype"]), tuple(meta["shape"])
        if mmap and meta["nbytes"]:
            arrays[name] = np.memmap(path, dtype=dt, mode="r", offset=meta["offset"], shape=shape)
        else:
            with open(path, "rb") as f:
                f.seek(meta["offset"])
                arrays[name] = np.frombuffer(f.read(meta["nbytes"]), dtype=dt).reshape(shape).copy()
    return Bundle(head["config"], arrays, head.get("source", {}))


def write_bundle(path: str | Path, config: dict, arrays: dict, source: dict | None = None) -> Path:
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    arrs = {k: np.ascontiguousarray(v) for k, v in arrays.items()}
    meta = {k: {"dtype": a.dtype.str, "shape": list(a.shape), "offset": 0, "nbytes": int(a.nbytes)}
            for k, a in arrs.items()}
    while True:  # offsets change the header length; iterate to a fixed point
        header = json.dumps({"version": VERSION, "config": config, "arrays": meta, "source": source or {}},
                            sort_keys=True).encode("utf-8")
        offset = _align(16 + len(header) + 256)
        placed = {}
        for k, a in arrs.items():
            placed[k] = dict(meta[k], offset=offset)
            offset = _align(offset + a.nbytes)
        if placed == meta:
            break
        meta = placed
    with open(path, "wb") as f:
        f.write(MAGIC)
        f.write(struct.pack("<Q", len(header)))
        f.write(header)
        for k, a in arrs.items():
            f.write(b"\0" * (meta[k]["offset"] - f.tell()))
            a.astype(a.dtype.newbyteorder("<"), copy=False).tofile(f)
    return path


def as_bundle(bundle) -> Bundle:
    """A Bundle from a Bundle, a path, or any object with ``config`` and ``arrays`` (the reference's
    own ``drafting.export_drafter.Bundle`` included)."""
    if isinstance(bundle, (str, Path)):
        return load_bundle(bundle)
    if isinstance(bundle, Bundle):
        return bundle
    return Bundle(dict(bundle.config), dict(bundle.arrays), dict(getattr(bundle, "source", {}) or {}))
