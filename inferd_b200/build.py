"""Build libinferd_sm100a.so from inferd_b200/csrc with nvcc (sm_100a only), and the small
host-side extension module _hostops (page-table loops, CPython C API) with g++.

The library is a plain C-ABI shared object (no torch symbols), built in-tree into
inferd_b200/lib/ so it travels with the source tree.  Usage:

    python -m inferd_b200.build            # build if any source is newer than the .so
    python -m inferd_b200.build --force
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
import sysconfig
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
LIB_DIR = PKG_DIR / "lib"
LIB_PATH = LIB_DIR / "libinferd_sm100a.so"
INCLUDE_DIR = REPO_DIR / "include"

SOURCES = ["runtime.cu", "cache_ops.cu", "paged_attention.cu", "paged_attention_noalloc.cu",
           "fp8_linear.cu", "sampling.cu", "peer.cu"]
HOSTOPS_SRC = CSRC / "host_ops.cpp"
HOSTOPS_PATH = PKG_DIR / ("_hostops" + (sysconfig.get_config_var("EXT_SUFFIX") or ".so"))

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
]


def nvcc_path() -> str:
    cand = shutil.which("nvcc")
    if cand:
        return cand
    for root in (os.environ.get("CUDA_HOME"), "/usr/local/cuda"):
        if root and Path(root, "bin", "nvcc").exists():
            return str(Path(root, "bin", "nvcc"))
    raise RuntimeError("nvcc not found; the inferd_b200 kernels need the CUDA toolkit to build")


def _sources() -> list[Path]:
    return [CSRC / s for s in SOURCES if (CSRC / s).exists()]


def _inputs() -> list[Path]:
    return _sources() + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE_DIR.glob("*.h")) + [Path(__file__)]


def build_hostops(force: bool = False) -> Path:
    """Compile the _hostops extension module in place (g++, CPython headers)."""
    if (not force and HOSTOPS_PATH.exists()
            and HOSTOPS_PATH.stat().st_mtime >= max(HOSTOPS_SRC.stat().st_mtime, Path(__file__).stat().st_mtime)):
        return HOSTOPS_PATH
    cxx = shutil.which("g++") or shutil.which("c++")
    if cxx is None:
        raise RuntimeError("g++ not found; the _hostops module needs a C++ compiler")
    tmp = HOSTOPS_PATH.with_name(HOSTOPS_PATH.name + ".tmp")
    cmd = [cxx, "-O2", "-std=c++17", "-shared", "-fPIC", "-fvisibility=hidden",
           f"-I{sysconfig.get_paths()['include']}", str(HOSTOPS_SRC), "-o", str(tmp)]
    proc = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)
    if proc.returncode != 0:
        raise RuntimeError(f"g++ failed:\n{proc.stdout.decode(errors='replace')}")
    os.replace(tmp, HOSTOPS_PATH)
    return HOSTOPS_PATH


def needs_build() -> bool:
    if not LIB_PATH.exists():
        return True
    lib_mtime = LIB_PATH.stat().st_mtime
    return any(p.stat().st_mtime > lib_mtime for p in _inputs())


def build(force: bool = False, verbose: bool = False, jobs: int | None = None) -> Path:
    """Compile every .cu to an object for sm_100a and link the shared library; build the
    _hostops module."""
    build_hostops(force=force)
    if not force and not needs_build():
        return LIB_PATH
    nvcc = nvcc_path()
    obj_dir = PKG_DIR / "_build"
    obj_dir.mkdir(exist_ok=True)
    LIB_DIR.mkdir(exist_ok=True)
    objs = []
    procs = []
    for src in _sources():
        obj = obj_dir / (src.stem + ".o")
        objs.append(obj)
        cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, f"-I{INCLUDE_DIR}", "-c", str(src), "-o", str(obj)]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
            print(" ".join(cmd), flush=True)
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
    failed = []
    for src, proc in procs:
        out, _ = proc.communicate()
        text = out.decode(errors="replace")
        if proc.returncode != 0:
            failed.append((src, text))
        elif verbose and text:
            print(text)
    if failed:
        msg = "\n".join(f"--- {src.name}\n{text}" for src, text in failed)
        raise RuntimeError(f"nvcc failed:\n{msg}")
    tmp = LIB_PATH.with_suffix(".so.tmp")
    link = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objs), "-lcudart"]
    subprocess.run(link, check=True)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true", help="print nvcc commands and -Xptxas -v")
    args = ap.parse_args(argv)
    path = build(force=args.force, verbose=args.verbose)
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
