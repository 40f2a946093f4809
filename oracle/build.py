"""Build recipe for the oracle's native pieces (TEST INFRASTRUCTURE ONLY).

* ``oracle/_build/libngram_index.so`` from ``oracle/ngram_index.c`` (plain C restatement of the
  integer addressing) -- always built.
* ``oracle/_ref/morbius_cpu_drafter*.so`` -- the reference's own C++ CPU drafter, compiled with
  g++ directly from its single source file where it lies in the reference checkout
  (``drafting/cpu/drafter.cpp``; the reference builds it as a torch CppExtension,
  ``drafting/cpu/setup.py:17-27``).  Built only when the reference checkout is present; the
  reference sources are never copied.  ``-O3 -march=x86-64-v3`` replaces the reference's
  ``-march=native`` so the library runs on any AVX2 host it travels to.

Usage: ``python oracle/build.py [--reference PATH]``; outputs are git-ignored.
"""

from __future__ import annotations

import argparse
import os
import subprocess
import sys
import sysconfig
from pathlib import Path

HERE = Path(__file__).resolve().parent
BUILD = HERE / "_build"
REF_OUT = HERE / "_ref"
# the reference checkout: LNGRAM_REFERENCE, else a directory named "reference" beside this repository
DEFAULT_REFERENCE = Path(os.environ.get("LNGRAM_REFERENCE") or (HERE.parent.parent / "reference"))


def _run(cmd: list) -> None:
    subprocess.run(cmd, check=True)


def build_c_oracle() -> Path:
    BUILD.mkdir(exist_ok=True)
    out = BUILD / "libngram_index.so"
    src = HERE / "ngram_index.c"
    if not out.exists() or out.stat().st_mtime < src.stat().st_mtime:
        _run(["gcc", "-O2", "-shared", "-fPIC", "-o", str(out), str(src)])
    return out


def load_c_oracle():
    """ctypes handle of the C oracle with its argument types declared."""
    import ctypes as C

    lib = C.CDLL(str(build_c_oracle()))
    lib.oracle_pack_codes.argtypes = [C.c_void_p, C.c_int64, C.c_int64, C.c_int, C.c_void_p]
    lib.oracle_pack_codes.restype = C.c_int
    lib.oracle_row_indices.argtypes = [C.c_void_p, C.c_int64, C.c_int64, C.c_int64, C.c_int, C.c_int, C.c_void_p,
                                       C.c_void_p, C.c_void_p]
    lib.oracle_row_indices.restype = C.c_int
    return lib


def ref_drafter_path() -> Path:
    return REF_OUT / ("morbius_cpu_drafter" + sysconfig.get_config_var("EXT_SUFFIX"))


def build_reference_drafter(reference: Path = DEFAULT_REFERENCE) -> Path | None:
    src = reference / "drafting" / "cpu" / "drafter.cpp"
    if not src.exists():
        return None
    out = ref_drafter_path()
    if out.exists() and out.stat().st_mtime >= src.stat().st_mtime:
        return out
    import torch
    from torch.utils import cpp_extension as ce

    REF_OUT.mkdir(exist_ok=True)
    inc = [f"-I{p}" for p in ce.include_paths()] + [f"-I{sysconfig.get_paths()['include']}"]
    libdir = ce.library_paths()[0]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = (["g++", "-O3", "-march=x86-64-v3", "-std=c++17", "-shared", "-fPIC",
            "-DTORCH_EXTENSION_NAME=morbius_cpu_drafter", "-DTORCH_API_INCLUDE_EXTENSION_H",
            f"-D_GLIBCXX_USE_CXX11_ABI={abi}"] + inc + [str(src), "-o", str(out), f"-L{libdir}",
           f"-Wl,-rpath,{libdir}", "-lc10", "-ltorch", "-ltorch_cpu", "-ltorch_python"])
    _run(cmd)
    return out


def load_reference_drafter():
    """Import the prebuilt reference drafter module (None when it was not built)."""
    path = ref_drafter_path()
    if not path.exists():
        return None
    import importlib.util

    import torch  # noqa: F401  (loads libtorch before the extension)

    spec = importlib.util.spec_from_file_location("morbius_cpu_drafter", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--reference", type=Path, default=DEFAULT_REFERENCE)
    args = ap.parse_args(argv)
    print(build_c_oracle())
    print(build_reference_drafter(args.reference))


if __name__ == "__main__":
    sys.exit(main())
