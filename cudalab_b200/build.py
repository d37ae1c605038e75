"""Build (or reuse) the sm_100a shared library and hand out operator extensions.

Mirrors the role of the reference's `cudalab/build.py:build(op)`
(cudalab/build.py:72-114): `build("int4gemv")` / `build("qgemv")` return an
object exposing `forward / forward_into / native_timing / variants /
all_variants / quarantined_variants`, the duck-typed `ext` the correctness,
negative and benchmark suites drive.

Differences by design:
  * one C-ABI shared library, `cudalab_b200/_lib/libcudalab_gemv.so`, compiled
    in-tree by nvcc for `compute_100a/sm_100a` (no torch extension, no JIT
    cache under the home directory), loaded with ctypes;
  * no `--use_fast_math` (the GEMV needs none and it would change division);
  * rebuilt when the SHA-256 of the sources + flags changes (stamp file next
    to the library).
"""
from __future__ import annotations

import hashlib
import json
import os
import shutil
import subprocess
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB_DIR = PKG / "_lib"
LIB_PATH = LIB_DIR / "libcudalab_gemv.so"
STAMP = LIB_DIR / "libcudalab_gemv.stamp.json"
HEADER = ROOT / "include" / "cudalab_gemv.h"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
# --split-compile 0: the optimiser and ptxas work on a translation unit's
# kernels in parallel on every host core (the kernel unit holds dozens of
# template instantiations)
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--split-compile", "0"]
SOURCES = ["gemv_kernels.cu", "gemv_dense.cu", "quantize.cu", "capi.cu"]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found: cannot build libcudalab_gemv.so")
    return cand


def _fingerprint() -> str:
    h = hashlib.sha256()
    files = sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h"))
    files.append(HEADER)
    for f in files:
        h.update(f.name.encode())
        h.update(f.read_bytes())
    h.update(" ".join(ARCH_FLAGS + NVCC_FLAGS).encode())
    return h.hexdigest()[:16]


def library_is_current() -> bool:
    if not LIB_PATH.exists() or not STAMP.exists():
        return False
    try:
        return json.loads(STAMP.read_text()).get("hash") == _fingerprint()
    except (OSError, ValueError):
        return False


def build_library(force: bool = False, verbose: bool = False) -> Path:
    """Compile libcudalab_gemv.so in-tree unless an up-to-date build exists."""
    if not force and library_is_current():
        return LIB_PATH
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    obj_dir = LIB_DIR / "obj"
    obj_dir.mkdir(exist_ok=True)
    tmp = LIB_PATH.with_suffix(".so.tmp")
    nvcc = _nvcc()
    # every translation unit compiles concurrently, then one link
    jobs = []
    for src in SOURCES:
        cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, "-c", str(CSRC / src),
               "-o", str(obj_dir / (Path(src).stem + ".o"))]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
            print(" ".join(cmd))
        jobs.append(subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT,
                                     text=True))
    logs = [(src, p.communicate()[0], p.returncode) for src, p in zip(SOURCES, jobs)]
    failed = [(src, out) for src, out, rc in logs if rc != 0]
    if failed:
        raise RuntimeError("nvcc failed:\n" + "\n".join(f"{s}:\n{o}" for s, o in failed))
    if verbose:
        for _, out, _ in logs:
            print(out)
    link = [nvcc, *ARCH_FLAGS, "-shared",
            *[str(obj_dir / (Path(s).stem + ".o")) for s in SOURCES], "-o", str(tmp)]
    proc = subprocess.run(link, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError("nvcc link failed:\n" + proc.stdout + proc.stderr)
    os.replace(tmp, LIB_PATH)
    STAMP.write_text(json.dumps({"hash": _fingerprint(), "sources": SOURCES,
                                 "flags": ARCH_FLAGS + NVCC_FLAGS}, indent=2))
    return LIB_PATH


def build(op: str = "int4gemv", force: bool = False, verbose: bool = False):
    """Return the extension object of operator `op` ("int4gemv" | "qgemv" | "gemv")."""
    build_library(force=force, verbose=verbose)
    from .ext import get_ext
    return get_ext(op)


if __name__ == "__main__":
    import sys
    p = build_library(force="--force" in sys.argv, verbose=True)
    print(p)
