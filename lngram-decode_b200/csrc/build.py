"""Build ``liblngram_b200.so`` (the C-ABI library) in-tree for sm_100a with nvcc.

    python lngram-decode_b200/csrc/build.py [--force] [--verbose]

The library is one translation unit (``lngram_b200.cu`` includes every kernel header), built
with ``-gencode arch=compute_100a,code=sm_100a -lineinfo -O3``.  A stamp of the source hashes
skips rebuilding when nothing changed.  The output is git-ignored and travels with the
repository snapshot to the GPU box.
"""

from __future__ import annotations

import argparse
import hashlib
import os
import shutil
import subprocess
import sys
from pathlib import Path

CSRC = Path(__file__).resolve().parent
PKG = CSRC.parent
REPO = PKG.parent
LIB = PKG / "liblngram_b200.so"
STAMP = PKG / ".liblngram_b200.stamp"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + [REPO / "include" / "lngram_b200.h"]


def _digest(flags: list[str]) -> str:
    h = hashlib.sha256()
    for p in _sources():
        h.update(p.name.encode())
        h.update(p.read_bytes())
    h.update(" ".join(flags).encode())
    return h.hexdigest()


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found: the lngram_b200 CUDA library cannot be built")
    return cand


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> Path:
    flags = ARCH + ["-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-shared", "-diag-suppress", "177"]
    if ptxas_info:
        flags += ["-Xptxas", "-v"]
    digest = _digest(flags)
    if not force and LIB.exists() and STAMP.exists() and STAMP.read_text().strip() == digest:
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc()] + flags + ["-o", str(tmp), str(CSRC / "lngram_b200.cu")]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    out = (res.stdout or "") + (res.stderr or "")
    out = "\n".join(l for l in out.splitlines() if "Warning: The 'compute_" not in l)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{out}")
    if verbose or ptxas_info:
        print(out)
    os.replace(tmp, LIB)
    STAMP.write_text(digest)
    return LIB


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print registers / spills / shared memory per kernel")
    args = ap.parse_args(argv)
    print(build(args.force, args.verbose, args.ptxas_info))
    return 0


if __name__ == "__main__":
    sys.exit(main())
