"""Build the sm_100a shared library behind the C ABI (``include/vggt_b200.h``).

Every ``csrc/*.cu`` file is compiled by nvcc for ``sm_100a`` only and linked into
``_lib/libvggt_b200.so`` inside the package, so the library travels with the source tree.
Objects are rebuilt only when a source or header is newer than the object.

Usage: ``python 4d_ttt_merging_b200/build.py [--force] [--verbose]``.
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
OUT_DIR = PKG_DIR / "_lib"
OBJ_DIR = PKG_DIR / "_build"
LIB_NAME = "libvggt_b200.so"
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-fvisibility=hidden",
    "-I", str(REPO_DIR / "include"),
]


def _nvcc() -> str:
    for candidate in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if candidate and (Path(candidate).exists() or candidate == "nvcc"):
            return candidate
    raise RuntimeError("nvcc not found")


def library_path() -> Path:
    return OUT_DIR / LIB_NAME


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + [REPO_DIR / "include" / "vggt_b200.h"]


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile every CUDA source for sm_100a and link the shared library; return its path."""
    nvcc = _nvcc()
    OUT_DIR.mkdir(exist_ok=True)
    OBJ_DIR.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    headers = _headers()
    jobs = []
    for src in sources:
        obj = OBJ_DIR / (src.stem + ".o")
        if force or _stale(obj, [src, *headers]):
            cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
            if verbose:
                cmd.insert(1, "-Xptxas=-v")
            jobs.append((src, cmd))

    def run(job):
        src, cmd = job
        proc = subprocess.run(cmd, capture_output=True, text=True)
        return src, proc

    failures = []
    with ThreadPoolExecutor(max_workers=max(1, min(len(jobs), os.cpu_count() or 1))) as pool:
        for src, proc in pool.map(run, jobs):
            if verbose and (proc.stdout or proc.stderr):
                sys.stderr.write(proc.stdout + proc.stderr)
            if proc.returncode != 0:
                failures.append((src, proc.stdout + proc.stderr))
    if failures:
        msg = "\n".join(f"--- {s.name} ---\n{out}" for s, out in failures)
        raise RuntimeError(f"nvcc failed:\n{msg}")
    objs = [OBJ_DIR / (s.stem + ".o") for s in sources]
    lib = library_path()
    if force or jobs or _stale(lib, objs):
        cmd = [nvcc, *ARCH_FLAGS, "-shared", "-Xcompiler", "-fPIC", "-o", str(lib), *map(str, objs)]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"link failed:\n{proc.stdout}{proc.stderr}")
    return lib


if __name__ == "__main__":
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose))
