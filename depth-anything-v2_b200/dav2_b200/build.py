"""Build libdav2_b200.so in-tree: every .cu compiled by nvcc for sm_100a
(-gencode arch=compute_100a,code=sm_100a), the C++ runtime by g++, linked
into depth-anything-v2_b200/lib/libdav2_b200.so."""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent.parent
CSRC = PKG / "csrc"
ROOT = PKG.parent
BUILD = PKG / "_build"
LIB = PKG / "lib" / "libdav2_b200.so"
CUDA = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA / "bin" / "nvcc")
CXX = "/usr/bin/g++" if Path("/usr/bin/g++").exists() else "g++"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
                     "--expt-relaxed-constexpr", "-ccbin", CXX,
                     f"-I{ROOT / 'include'}", f"-I{CSRC}", f"-I{CSRC / 'runtime'}"]
CXX_FLAGS = ["-O2", "-std=c++17", "-fPIC", "-fvisibility=hidden", "-Wall", "-Wextra", "-Wno-unused-parameter",
             f"-I{ROOT / 'include'}", f"-I{CSRC}", f"-I{CSRC / 'runtime'}", f"-I{CUDA / 'include'}"]


def _sources():
    cu = sorted(CSRC.glob("*.cu")) + sorted((CSRC / "runtime").glob("*.cu"))
    cpp = sorted((CSRC / "runtime").glob("*.cpp"))
    return cu, cpp


def _needs(obj: Path, src: Path, deps) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return src.stat().st_mtime > t or any(d.stat().st_mtime > t for d in deps)


def build(verbose: bool = False, jobs: int | None = None) -> Path:
    BUILD.mkdir(exist_ok=True)
    LIB.parent.mkdir(exist_ok=True)
    cu, cpp = _sources()
    headers = (list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list((CSRC / "runtime").glob("*.h")) +
               list((ROOT / "include").glob("*.h")))
    cmds = []
    objs = []
    for src in cu:
        obj = BUILD / (src.stem + ".cu.o")
        objs.append(obj)
        if _needs(obj, src, headers):
            cmds.append([NVCC, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)])
    for src in cpp:
        obj = BUILD / (src.stem + ".o")
        objs.append(obj)
        if _needs(obj, src, headers):
            cmds.append([CXX, *CXX_FLAGS, "-c", str(src), "-o", str(obj)])

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"compile failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        if verbose and (r.stderr.strip()):
            print(r.stderr, flush=True)
        return r

    with ThreadPoolExecutor(max_workers=jobs or os.cpu_count() or 4) as ex:
        list(ex.map(run, cmds))
    if cmds or not LIB.exists():
        link = [NVCC, *ARCH, "-shared", "-ccbin", CXX, "-o", str(LIB), *map(str, objs),
                "-lcudart", "-ldl", "-lpthread"]
        run(link)
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
