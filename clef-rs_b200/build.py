"""Builds libclef_b200.so in place: every csrc/*.cu compiled for sm_100a.

    python clef-rs_b200/build.py [--jobs N] [--verbose]

Objects go to clef-rs_b200/_build/; the shared library to
clef-rs_b200/libclef_b200.so. nvcc cross-compiles without a GPU.
"""
import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
OUT = HERE / "libclef_b200.so"
BUILD = HERE / "_build"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3",
         "--expt-relaxed-constexpr", "-Xptxas", "-v", "-I", str(HERE.parent / "include")]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if c and Path(c).exists():
            return c
    raise RuntimeError("nvcc not found")


def host_cxx() -> list:
    # Use the system g++ as nvcc's host compiler (a CXX from the environment
    # may be a wrapper without the OpenMP/C++ spec files).
    return ["-ccbin", "/usr/bin/g++"] if Path("/usr/bin/g++").exists() else []


def compile_one(src: Path, verbose: bool) -> tuple:
    obj = BUILD / (src.stem + ".o")
    log = BUILD / (src.stem + ".ptxas.txt")
    deps = [src] + list(CSRC.glob("*.cuh")) + [HERE.parent / "include" / "clef_b200.h"]
    if obj.exists() and all(obj.stat().st_mtime >= d.stat().st_mtime for d in deps):
        return src.name, True, ""
    cmd = [nvcc()] + host_cxx() + ARCH + FLAGS + ["-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    log.write_text(r.stdout + r.stderr)
    if verbose or r.returncode:
        return src.name, r.returncode == 0, r.stdout + r.stderr
    return src.name, True, ""


def build(jobs: int = 8, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        results = list(ex.map(lambda s: compile_one(s, verbose), srcs))
    failed = [r for r in results if not r[1]]
    for name, ok, out in results:
        if out:
            print(f"== {name}\n{out}", file=sys.stderr)
    if failed:
        raise RuntimeError("nvcc failed: " + ", ".join(r[0] for r in failed))
    objs = [str(BUILD / (s.stem + ".o")) for s in srcs]
    newest = max(Path(o).stat().st_mtime for o in objs)
    if not OUT.exists() or OUT.stat().st_mtime < newest:
        cmd = [nvcc()] + host_cxx() + ARCH + ["-shared", "-o", str(OUT)] + objs
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode:
            raise RuntimeError("link failed:\n" + r.stdout + r.stderr)
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--jobs", type=int, default=8)
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(a.jobs, a.verbose))
