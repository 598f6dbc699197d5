"""Build the in-tree sm_100a shared library (libb200attn.so) and the C++ harness
binaries with nvcc.  Everything is compiled for `-gencode arch=compute_100a,code=sm_100a`
only; the artefacts land next to this file so they travel with the source tree.

Usage: python -m benchmark_b200.build [--verbose] [--ptxas-info]
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
LIB = PKG / "libb200attn.so"
HARNESS_SRC = PKG / "harness"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
          f"-I{INCLUDE}", f"-I{CSRC}"]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; the sm_100a build needs the CUDA toolkit")
    return cand


def _run(cmd: list[str], verbose: bool) -> str:
    if verbose:
        print(" ".join(cmd), flush=True)
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        sys.stderr.write(proc.stdout + proc.stderr)
        raise RuntimeError(f"build step failed: {' '.join(cmd[:3])} ...")
    return proc.stdout + proc.stderr


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def lib_sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + [INCLUDE / "b200attn.h"]


def build_lib(verbose: bool = False, ptxas_info: bool = False, force: bool = False) -> Path:
    if not force and not ptxas_info and not _stale(LIB, lib_sources()):
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, *COMMON, "-shared", "-o", str(tmp), str(CSRC / "b200attn.cu"),
           "-lcublas"]
    if ptxas_info:
        cmd.insert(1, "-Xptxas=-v")
    out = _run(cmd, verbose)
    if ptxas_info:
        print(out)
    os.replace(tmp, LIB)
    return LIB


def build_harness(verbose: bool = False, force: bool = False) -> list[Path]:
    built = []
    if not HARNESS_SRC.exists():
        return built
    common_h = sorted(HARNESS_SRC.glob("*.h")) + [INCLUDE / "b200attn.h"]
    for src in sorted(HARNESS_SRC.glob("*.cpp")):
        exe = PKG / "bin" / src.stem
        exe.parent.mkdir(exist_ok=True)
        if not force and not _stale(exe, [src, LIB, *common_h]):
            built.append(exe)
            continue
        cmd = [nvcc(), "-O2", "-std=c++17", f"-I{INCLUDE}", f"-I{HARNESS_SRC}",
               "-o", str(exe), str(src),
               f"-L{PKG}", "-lb200attn", f"-Xlinker=-rpath,$ORIGIN/..", "-lcudart", "-lpthread"]
        _run(cmd, verbose)
        built.append(exe)
    # Device-code tools (the peak probes): sm_100a, self-contained.
    csrc_h = sorted(CSRC.glob("*.cuh"))
    for src in sorted(HARNESS_SRC.glob("*.cu")):
        exe = PKG / "bin" / src.stem
        exe.parent.mkdir(exist_ok=True)
        if not force and not _stale(exe, [src, *csrc_h]):
            built.append(exe)
            continue
        cmd = [nvcc(), *ARCH, "-O3", "-std=c++17", "-lineinfo", f"-I{CSRC}", f"-I{INCLUDE}",
               "-o", str(exe), str(src), "-lcudart"]
        _run(cmd, verbose)
        built.append(exe)
    return built


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build_lib(a.verbose, a.ptxas_info, a.force))
    for exe in build_harness(a.verbose, a.force):
        print(exe)


if __name__ == "__main__":
    main()
