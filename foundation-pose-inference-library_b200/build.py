"""Build libfoundation_pose_nvidia.so (sm_100a) in-tree.

Compiles every csrc/*.cu and csrc/*.cpp with nvcc for sm_100a only and links
them into lib/libfoundation_pose_nvidia.so next to this file. Objects go to
_build/ at the repository root. Incremental: a source is recompiled when it or
any header under csrc/ or include/ is newer than its object.

Usage: python build.py [-j N] [--force]
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
OBJ = ROOT / "_build" / "fp"
LIB = PKG / "lib" / "libfoundation_pose_nvidia.so"

NVCC = os.environ.get("NVCC", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-std=c++20", "-O3", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden",
          "-DFOUNDATION_POSE_NVIDIA_EXPORTS", f"-I{INCLUDE}", f"-I{CSRC}"]


def sources() -> list[Path]:
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cpp")))


def newest_header() -> float:
    hdrs = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.hpp")) + list(CSRC.glob("*.h"))
    hdrs += list(INCLUDE.rglob("*.h")) + list(INCLUDE.rglob("*.hpp"))
    return max((h.stat().st_mtime for h in hdrs), default=0.0)


def compile_one(src: Path, force: bool, hdr_time: float) -> Path:
    obj = OBJ / (src.name + ".o")
    if not force and obj.exists():
        t = obj.stat().st_mtime
        if t >= src.stat().st_mtime and t >= hdr_time:
            return obj
    cmd = [NVCC, *ARCH, *COMMON, "-c", str(src), "-o", str(obj)]
    if src.suffix == ".cu":
        cmd += ["--expt-relaxed-constexpr"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
    return obj


def build(force: bool = False, jobs: int | None = None) -> Path:
    OBJ.mkdir(parents=True, exist_ok=True)
    LIB.parent.mkdir(parents=True, exist_ok=True)
    hdr_time = newest_header()
    srcs = sources()
    with cf.ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: compile_one(s, force, hdr_time), srcs))
    if force or not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        cmd = [NVCC, *ARCH, "-shared", "-o", str(LIB), *map(str, objs),
               "-lcudart", "-Xlinker", "-soname=libfoundation_pose_nvidia.so.1",
               "-Xlinker", "-z,defs"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    # Programs linked against the library record its soname (SOVERSION 1, as
    # the reference's CMake build sets it); the loader resolves that name.
    soname = LIB.with_name(LIB.name + ".1")
    if not soname.is_symlink() or os.readlink(soname) != LIB.name:
        if soname.exists() or soname.is_symlink():
            soname.unlink()
        soname.symlink_to(LIB.name)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("-j", type=int, default=None)
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args()
    try:
        print(build(args.force, args.j))
    except RuntimeError as e:
        print(e, file=sys.stderr)
        sys.exit(1)
