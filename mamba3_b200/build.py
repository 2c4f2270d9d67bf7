"""Build ``libmamba3_b200.so`` in-tree with nvcc for sm_100a.

    python -m mamba3_b200.build [--verbose]

The library has no dependency on torch headers: it is plain CUDA C++ behind the
C ABI of ``include/mamba3_b200.h``.  The result lands next to this file so that
it travels with the source tree.
"""

from __future__ import annotations

import hashlib
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libmamba3_b200.so"
# sha256 of the flags and every source the library was built from, written beside it
DIGEST = PKG / "libmamba3_b200.so.digest"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-I", str(ROOT / "include"),
]


def nvcc_path():
    for c in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and Path(c).exists():
            return c
    raise RuntimeError("nvcc not found")


def sources():
    return sorted(CSRC.glob("*.cu"))


def _deps():
    return sources() + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + [ROOT / "include" / "mamba3_b200.h"]


def source_digest() -> str:
    """sha256 over the compiler flags and the contents of every file the library is built from."""
    h = hashlib.sha256()
    h.update("\0".join(NVCC_FLAGS[:-1]).encode())  # the include path itself is machine-specific
    for p in _deps():
        h.update(p.relative_to(ROOT).as_posix().encode() + b"\0")
        h.update(p.read_bytes())
    return h.hexdigest()


def is_current() -> bool:
    """True when the library exists and was built from exactly the sources and flags present now."""
    try:
        return LIB.exists() and DIGEST.read_text().strip() == source_digest()
    except OSError:
        return False


def build(verbose: bool = False, force: bool = False, ptxas_verbose: bool = False) -> Path:
    """Compile the library unless it is current (same sources and flags, by content, not by mtime)."""
    srcs = sources()
    digest = source_digest()
    if not force and is_current():
        return LIB
    objdir = ROOT / "_build"
    objdir.mkdir(exist_ok=True)
    nvcc = nvcc_path()
    objs = []
    procs = []
    for s in srcs:
        o = objdir / (s.stem + ".o")
        cmd = [nvcc, *NVCC_FLAGS, "-c", str(s), "-o", str(o)]
        if ptxas_verbose:
            cmd += ["-Xptxas", "-v"]
        if verbose:
            print(" ".join(cmd))
        procs.append((s, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)))
        objs.append(o)
    failed = []
    for s, p in procs:
        out, _ = p.communicate()
        if verbose or ptxas_verbose or p.returncode != 0:
            sys.stdout.write(out)
        if p.returncode != 0:
            failed.append(s.name)
    if failed:
        raise RuntimeError(f"nvcc failed for {failed}")
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", *map(str, objs), "-o", str(tmp)]
    if verbose:
        print(" ".join(cmd))
    subprocess.check_call(cmd)
    os.replace(tmp, LIB)
    DIGEST.write_text(digest + "\n")
    return LIB


if __name__ == "__main__":
    build(verbose="--verbose" in sys.argv, force=True, ptxas_verbose="--ptxas" in sys.argv)
    print(LIB)
