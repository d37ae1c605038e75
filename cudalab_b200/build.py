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


# ---- the torch binding of the success path (csrc/torch_fast.cpp) ----
BINDING_SRC = CSRC / "torch_fast.cpp"
BINDING_NAME = "_cl_torch"
BINDING_STAMP = LIB_DIR / f"{BINDING_NAME}.stamp.json"


def binding_path() -> Path:
    import sysconfig
    return LIB_DIR / (BINDING_NAME + sysconfig.get_config_var("EXT_SUFFIX"))


def _binding_cmd(out: Path) -> list[str]:
    import sysconfig
    import torch
    from torch.utils import cpp_extension as ce
    inc = ce.include_paths("cuda") + [sysconfig.get_paths()["include"]]
    torch_lib = ce.library_paths("cuda")[0]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    return (["g++", "-O2", "-std=c++17", "-fPIC", "-shared", str(BINDING_SRC), "-o", str(out),
             f"-DTORCH_EXTENSION_NAME={BINDING_NAME}", "-DTORCH_API_INCLUDE_EXTENSION_H",
             f"-D_GLIBCXX_USE_CXX11_ABI={abi}"]
            + [f"-I{p}" for p in inc]
            + [f"-L{torch_lib}", "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_python",
               f"-L{LIB_DIR}", "-lcudalab_gemv", "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{torch_lib}"])


def _binding_fingerprint() -> str:
    import torch
    h = hashlib.sha256()
    for f in (BINDING_SRC, HEADER):
        h.update(f.read_bytes())
    h.update(torch.__version__.encode())
    return h.hexdigest()[:16]


def build_binding(force: bool = False) -> Path:
    """Compile the torch binding (g++, torch headers) next to the library."""
    out = binding_path()
    fp = _binding_fingerprint()
    if not force and out.exists() and BINDING_STAMP.exists():
        try:
            if json.loads(BINDING_STAMP.read_text()).get("hash") == fp:
                return out
        except (OSError, ValueError):
            pass
    tmp = out.with_name(out.name + ".tmp")
    proc = subprocess.run(_binding_cmd(tmp), capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError("g++ failed on torch_fast.cpp:\n" + proc.stdout + proc.stderr)
    os.replace(tmp, out)
    BINDING_STAMP.write_text(json.dumps({"hash": fp}, indent=2))
    return out


def build(op: str = "int4gemv", force: bool = False, verbose: bool = False):
    """Return the extension object of operator `op` ("int4gemv" | "qgemv" | "gemv" |
    "rmsnorm")."""
    build_library(force=force, verbose=verbose)
    build_binding(force=force)
    from .ext import get_ext
    return get_ext(op)


if __name__ == "__main__":
    import sys
    p = build_library(force="--force" in sys.argv, verbose=True)
    print(p)
