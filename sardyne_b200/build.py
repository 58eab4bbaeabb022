"""Build libsardyne.so (the B200 drop-in) from sardyne_b200/csrc with nvcc for sm_100a.

    python -m sardyne_b200.build [-j N] [--force]

Objects go to sardyne_b200/_build/, the library to sardyne_b200/lib/libsardyne.so. Both are
git-ignored build outputs. nvcc cross-compiles without a GPU.
"""
import argparse
import concurrent.futures as cf
import os
import pathlib
import shutil
import subprocess
import sys

PKG = pathlib.Path(__file__).resolve().parent
REPO = PKG.parent
CSRC = PKG / "csrc"
OBJ = PKG / "_build"
LIB = PKG / "lib" / "libsardyne.so"
INCLUDE = REPO / "include"

NVCC = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CUDA_FLAGS = ARCH + ["-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC,-Wall", "--expt-relaxed-constexpr",
                     "-I", str(INCLUDE), "-I", str(CSRC)]
CXX_FLAGS = ["-O2", "-std=c++17", "-fPIC", "-Wall", "-Wextra", "-I", str(INCLUDE), "-I", str(CSRC)]


def _headers():
    return list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))


def _stale(src: pathlib.Path, obj: pathlib.Path, deps) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return src.stat().st_mtime > t or any(d.stat().st_mtime > t for d in deps)


def _compile(src: pathlib.Path, obj: pathlib.Path):
    if src.suffix == ".cu":
        cmd = [NVCC, *CUDA_FLAGS, "-c", str(src), "-o", str(obj)]
    else:
        cmd = ["g++", *CXX_FLAGS, "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"compile failed: {src.name}\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return src.name


def build(jobs: int = 0, force: bool = False, verbose: bool = True) -> pathlib.Path:
    OBJ.mkdir(exist_ok=True)
    LIB.parent.mkdir(exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cpp"))
    deps = _headers()
    todo = [(s, OBJ / (s.stem + ".o")) for s in srcs]
    stale = [(s, o) for s, o in todo if force or _stale(s, o, deps)]
    jobs = jobs or min(len(stale) or 1, os.cpu_count() or 4)
    if stale:
        with cf.ThreadPoolExecutor(jobs) as ex:
            for name in ex.map(lambda so: _compile(*so), stale):
                if verbose:
                    print(f"  built {name}", file=sys.stderr)
    objs = [str(o) for _, o in todo]
    if stale or not LIB.exists():
        cmd = [NVCC, *ARCH, "-shared", "-o", str(LIB), *objs, "-lcuda"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        if verbose:
            print(f"  linked {LIB}", file=sys.stderr)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("-j", type=int, default=0)
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(a.j, a.force))
