"""Build recipe for the in-tree C-ABI library ``vlcache_b200/libvlcache_b200.so``.

Compiles every CUDA translation unit for sm_100a only (tcgen05/TMA code does not
exist on other architectures) with nvcc, links the host planner, and links the
CUDA runtime statically so the library has no torch dependency.  The driver API
(cuTensorMapEncodeTiled) is reached through cudaGetDriverEntryPoint, so the
library also loads on machines without a GPU (CPU-side tests use the planner).

Usage: ``python -m vlcache_b200.build [--force] [--verbose]``.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import hashlib
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
INCLUDE = REPO_DIR / "include"
BUILD_DIR = REPO_DIR / "_build" / "vlcache_b200"
LIB_PATH = PKG_DIR / "libvlcache_b200.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
CUDA_SOURCES = ["runtime.cu", "kv_ops.cu", "prefill_attn.cu", "decode_attn.cu", "metadata.cu", "gemm.cu", "content_hash.cu"]
CPP_SOURCES = ["plan.cpp"]


def nvcc_path() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; the vlcache_b200 CUDA library cannot be built")
    return cand


def _sources() -> list[Path]:
    return [CSRC / s for s in CUDA_SOURCES + CPP_SOURCES]


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


STAMP_PATH = LIB_PATH.with_name(LIB_PATH.name + ".srchash")


def source_hash() -> str:
    """SHA-256 over the bytes of every source, header and this recipe (names included):
    the library is rebuilt exactly when this differs from the hash it was built from."""
    h = hashlib.sha256()
    for p in _sources() + _headers() + [Path(__file__)]:
        h.update(p.name.encode())
        h.update(b"\0")
        h.update(p.read_bytes())
        h.update(b"\0")
    return h.hexdigest()


def is_fresh() -> bool:
    """True when the in-tree library exists and was built from the current sources."""
    return LIB_PATH.exists() and STAMP_PATH.exists() and STAMP_PATH.read_text().strip() == source_hash()


def _needs_build() -> bool:
    return not is_fresh()


def _compile(src: Path, verbose: bool) -> Path:
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    obj = BUILD_DIR / (src.name + ".o")
    cmd = [nvcc_path(), *ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
           "-I", str(INCLUDE), "-I", str(CSRC), "-c", str(src), "-o", str(obj)]
    if src.suffix == ".cu":
        # Relocatable device code: one library-wide device error word across units.
        cmd[1:1] = ["-rdc=true"] + (["-Xptxas", "-v"] if verbose else [])
    else:
        cmd += ["-x", "c++"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
    if verbose and (res.stdout or res.stderr):
        sys.stderr.write(res.stdout + res.stderr)
    return obj


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile (unless the library was built from exactly these sources) and return the
    path of the shared library."""
    if not force and not _needs_build():
        return LIB_PATH
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), _sources()))
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [nvcc_path(), *ARCH_FLAGS, "-rdc=true", "-shared", "-cudart", "static", "-Xcompiler", "-fPIC",
           "-o", str(tmp), *map(str, objs)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
    digest = source_hash()
    os.replace(tmp, LIB_PATH)
    STAMP_PATH.write_text(digest + "\n")
    return LIB_PATH


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true", help="print ptxas resource usage")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose))


if __name__ == "__main__":
    main()
