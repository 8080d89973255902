"""Build recipe for the in-tree C-ABI library ``tinyserve_b200/libtsb_moe.so``.

Compiles every ``csrc/*.cu`` for sm_100a with nvcc and links one shared
library.  Run ``python -m tinyserve_b200.build`` (or ``__graft_entry__.build()``).
Rebuild decisions are keyed on content, not timestamps: each object carries a
hash of its source, every header it can include and the compiler flags, and the
library a hash of its objects' keys, so an edited source is never served by a
stale library (and an unchanged tree is not rebuilt after a checkout).
"""
from __future__ import annotations

import hashlib
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
LIB = PKG / "libtsb_moe.so"
BUILD = PKG / "_build"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-Xptxas", "-v"] + ARCH + os.environ.get("TSB_NVCC_EXTRA", "").split()


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libtsb_moe.so")
    return cand


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _headers_digest() -> str:
    h = hashlib.sha256()
    for p in sorted(list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))):
        h.update(p.name.encode())
        h.update(p.read_bytes())
    return h.hexdigest()


def _obj_key(src: Path, headers: str) -> str:
    h = hashlib.sha256()
    h.update(src.read_bytes())
    h.update(headers.encode())
    h.update(" ".join(NVCC_FLAGS).encode())
    return h.hexdigest()


def _lib_key(keys: list[str]) -> str:
    return hashlib.sha256(("|".join(keys) + " ".join(ARCH)).encode()).hexdigest()


def _stamp(p: Path) -> Path:
    return p.with_name(p.name + ".key")


def _read(p: Path) -> str:
    return p.read_text().strip() if p.exists() else ""


def _stale() -> bool:
    if not LIB.exists():
        return True
    headers = _headers_digest()
    return _read(_stamp(LIB)) != _lib_key([_obj_key(s, headers) for s in sources()])


def build(force: bool = False, verbose: bool = False) -> Path:
    headers = _headers_digest()
    keys = [_obj_key(s, headers) for s in sources()]
    lib_key = _lib_key(keys)
    if not force and LIB.exists() and _read(_stamp(LIB)) == lib_key:
        return LIB
    BUILD.mkdir(exist_ok=True)
    nvcc = _nvcc()
    objs = []
    for src, key in zip(sources(), keys):
        obj = BUILD / (src.stem + ".o")
        objs.append(str(obj))
        if not force and obj.exists() and _read(_stamp(obj)) == key:
            continue
        cmd = [nvcc, *NVCC_FLAGS, "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if verbose or r.returncode:
            sys.stderr.write(r.stdout + r.stderr)
        if r.returncode:
            raise RuntimeError(f"nvcc failed on {src.name}")
        (BUILD / (src.stem + ".ptxas.txt")).write_text(r.stderr)
        _stamp(obj).write_text(key)
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc, "-shared", *ARCH, "-o", str(tmp), *objs, "-lcudart", "-ldl"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("link of libtsb_moe.so failed")
    os.replace(tmp, LIB)
    _stamp(LIB).write_text(lib_key)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
