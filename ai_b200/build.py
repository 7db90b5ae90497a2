"""Builds the sm_100a shared library ``ai_b200/libfgemma.so`` with nvcc.

The library is built in-tree so it travels with the repository snapshot;
every translation unit is compiled for ``sm_100a`` only (tcgen05 / TMA code
does not exist on other targets). Objects are cached under ``_build/`` and
rebuilt when a source or header is newer.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = ROOT / "_build" / "fgemma"
LIB = PKG / "libfgemma.so"

SOURCES = [
    "fg_runtime.cu",
    "fg_gemm.cu",
    "fg_elementwise.cu",
    "fg_attention.cu",
    "fg_attn_tc.cu",
    "fg_ops.cu",
    "fg_model.cu",
    "fg_noalloc.cu",
    "fg_multi.cu",
    "fg_cluster.cu",
]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler", "-fPIC",
    "-Xcompiler", "-O3",
    "--expt-relaxed-constexpr",
    "-Xptxas", "-v",
    "-I", str(ROOT / "include"),
]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(path).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libfgemma")
    return path


def _newest_header() -> float:
    hs = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list((ROOT / "include").glob("*.h"))
    return max((h.stat().st_mtime for h in hs), default=0.0)


def build(verbose: bool = False, jobs: int | None = None) -> Path:
    """Compiles every CUDA source for sm_100a and links libfgemma.so."""
    BUILD.mkdir(parents=True, exist_ok=True)
    hdr = _newest_header()
    objs = []
    procs = []
    for src in SOURCES:
        s = CSRC / src
        o = BUILD / (src + ".o")
        objs.append(o)
        if o.exists() and o.stat().st_mtime >= max(s.stat().st_mtime, hdr):
            continue
        cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-c", str(s), "-o", str(o)]
        log = open(BUILD / (src + ".log"), "w")
        procs.append((src, subprocess.Popen(cmd, stdout=log, stderr=subprocess.STDOUT), log))
    failed = []
    for src, p, log in procs:
        rc = p.wait()
        log.close()
        text = (BUILD / (src + ".log")).read_text()
        if verbose or rc != 0:
            sys.stderr.write(f"--- nvcc {src} (rc={rc})\n{text}\n")
        if rc != 0:
            failed.append(src)
    if failed:
        raise RuntimeError(f"nvcc failed for {failed}")
    newest_obj = max(o.stat().st_mtime for o in objs)
    if not LIB.exists() or LIB.stat().st_mtime < newest_obj:
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
