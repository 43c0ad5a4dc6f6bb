"""Build libaxq8.so (the C-ABI library) in-tree for sm_100a with nvcc.

Usage: python -m axion_b200.build [--force] [-j N]

Every ``axion_b200/csrc/*.cu`` / ``*.cpp`` is compiled to an object under
``axion_b200/_build/`` and linked into ``axion_b200/libaxq8.so``.  The CUDA
runtime is linked statically so the library does not depend on which
libcudart the host process (e.g. torch) has loaded; both share the device's
primary context, so device pointers and streams pass freely between them.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libaxq8.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-O3", "-Xptxas", "-O3",
    f"-I{ROOT / 'include'}", f"-I{CSRC}",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def nccl_include() -> list[str]:
    """NCCL header location and the directory of its library (torch's bundled
    NCCL, else the system one); the library is opened at run time."""
    try:
        import nvidia.nccl  # type: ignore
        root = Path(list(nvidia.nccl.__path__)[0])
        if (root / "include" / "nccl.h").exists():
            return [f"-I{root / 'include'}", f'-DAXQ8_NCCL_DIR="{root / "lib"}"']
    except Exception:
        pass
    return []


def sources() -> list[Path]:
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cpp")))


def _headers_mtime() -> float:
    hs = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list((ROOT / "include").glob("*.h"))
    return max((h.stat().st_mtime for h in hs), default=0.0)


def _compile(src: Path, force: bool, hdr_mtime: float) -> Path:
    obj = BUILD / (src.name + ".o")
    if (not force and obj.exists() and obj.stat().st_mtime >= src.stat().st_mtime
            and obj.stat().st_mtime >= hdr_mtime):
        return obj
    cmd = [nvcc(), *NVCC_FLAGS, *nccl_include(), "-c", str(src), "-o", str(obj)]
    if src.suffix == ".cpp":
        cmd[1:1] = ["-x", "cu"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
    return obj


def build(force: bool = False, jobs: int | None = None) -> Path:
    BUILD.mkdir(exist_ok=True)
    srcs = sources()
    hm = _headers_mtime()
    with cf.ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: _compile(s, force, hm), srcs))
    newest = max(o.stat().st_mtime for o in objs)
    if force or not LIB.exists() or LIB.stat().st_mtime < newest:
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(LIB), *map(str, objs), "-ldl"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


CPP_SRC = PKG / "cpp" / "axion_b200.cpp"
CPP_LIB = PKG / "libaxion_b200_cpp.so"


def build_cpp(ref_include: str | Path, force: bool = False) -> Path:
    """The C++ boundary (include/axion_b200.hpp) for the reference's runtime:
    compiled against the reference's own headers (its inference/cpp tree,
    `ref_include`), linked to libaxq8.so and the CUDA runtime.  The symbols of
    the reference's Tensor factory stay undefined here: the runtime that loads
    the library provides them."""
    ref_include = Path(ref_include)
    if not (ref_include / "core" / "tensor.hpp").exists():
        raise RuntimeError(f"reference headers not found under {ref_include}")
    lib = build()
    deps = [CPP_SRC, ROOT / "include" / "axion_b200.hpp", ROOT / "include" / "axq8.h", lib]
    if not force and CPP_LIB.exists() and CPP_LIB.stat().st_mtime >= max(
            d.stat().st_mtime for d in deps):
        return CPP_LIB
    cuda = Path(nvcc()).resolve().parent.parent
    cmd = ["g++", "-std=c++17", "-O2", "-fPIC", "-shared", "-o", str(CPP_LIB), str(CPP_SRC),
           f"-I{ROOT / 'include'}", f"-I{ref_include}", f"-I{cuda / 'include'}",
           f"-L{PKG}", "-laxq8", f"-L{cuda / 'lib64'}", "-lcudart",
           "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{cuda / 'lib64'}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"g++ failed for {CPP_SRC.name}:\n{r.stdout}\n{r.stderr}")
    return CPP_LIB


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=None)
    ap.add_argument("--cpp", metavar="REF_INCLUDE", default=None,
                    help="also build the C++ boundary against the reference's inference/cpp tree")
    args = ap.parse_args()
    print(build(args.force, args.j))
    if args.cpp:
        print(build_cpp(args.cpp, args.force))
    return 0


if __name__ == "__main__":
    sys.exit(main())
