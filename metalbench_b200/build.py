"""Build libmb200.so in-tree with nvcc for sm_100a.

    python -m metalbench_b200.build [--force] [--verbose]

Every ``csrc/*.cu`` is compiled with
``-gencode arch=compute_100a,code=sm_100a -lineinfo -O3`` into ``_build/`` and
linked (static cudart, NCCL from the torch-bundled wheel or the system) into
``metalbench_b200/libmb200.so``. Objects are rebuilt only when a source or
header is newer. No GPU is needed.
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
REPO = PKG.parent
CSRC = PKG / "csrc"
BUILD = REPO / "_build"
LIB = PKG / "libmb200.so"
HOST = PKG / "mb200_host"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-Xptxas", "-warn-spills"]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found (CUDA 12.9 toolkit expected at /usr/local/cuda)")
    return cand


def nccl_paths():
    """(include_dir, lib_dir) of an NCCL with headers and libnccl.so.2."""
    cands = []
    try:
        import nvidia.nccl as _n  # torch-bundled NCCL wheel
        root = Path(list(_n.__path__)[0])
        cands.append((root / "include", root / "lib"))
    except Exception:
        pass
    cands.append((Path("/usr/include"), Path("/usr/lib/x86_64-linux-gnu")))
    for inc, lib in cands:
        if (inc / "nccl.h").exists() and (lib / "libnccl.so.2").exists():
            return inc, lib
    return None, None


def _stale(obj: Path, deps) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    nvcc = _nvcc()
    BUILD.mkdir(exist_ok=True)
    headers = list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh")) + list((REPO / "include").glob("*.h"))
    sources = sorted(CSRC.glob("*.cu"))
    nccl_inc, nccl_lib = nccl_paths()
    inc = ["-I", str(REPO / "include"), "-I", str(CSRC)]
    if nccl_inc:
        inc += ["-I", str(nccl_inc), "-DMB_HAVE_NCCL=1"]

    def compile_one(src: Path):
        obj = BUILD / (src.stem + ".o")
        if not force and not _stale(obj, [src] + headers):
            return obj, None
        cmd = [nvcc, *ARCH, *NVCC_FLAGS, *inc, "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        p = subprocess.run(cmd, capture_output=True, text=True)
        if p.returncode != 0:
            return obj, f"{src.name}:\n{p.stdout}\n{p.stderr}"
        if verbose and p.stderr.strip():
            print(p.stderr, file=sys.stderr)
        return obj, None

    with cf.ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as ex:
        results = list(ex.map(compile_one, sources))
    errs = [e for _, e in results if e]
    if errs:
        raise RuntimeError("nvcc failed:\n" + "\n".join(errs))
    objs = [o for o, _ in results]
    if force or _stale(LIB, objs):
        link = [nvcc, *ARCH, "-shared", "-cudart", "static", "-o", str(LIB), *map(str, objs)]
        if nccl_lib:
            link += ["-L", str(nccl_lib), "-l:libnccl.so.2", "-Xlinker", f"-rpath={nccl_lib}"]
        link += ["-ldl", "-lpthread"]
        if verbose:
            print(" ".join(link), file=sys.stderr)
        p = subprocess.run(link, capture_output=True, text=True)
        if p.returncode != 0:
            raise RuntimeError(f"link failed:\n{p.stdout}\n{p.stderr}")
    host_src = PKG / "host" / "mb200_host.cpp"
    if force or _stale(HOST, [host_src, LIB] + headers):
        cmd = ["g++", "-O2", "-std=c++17", "-I", str(REPO / "include"), str(host_src), "-o",
               str(HOST), "-L", str(PKG), "-l:libmb200.so", "-Wl,-rpath,$ORIGIN"]
        p = subprocess.run(cmd, capture_output=True, text=True)
        if p.returncode != 0:
            raise RuntimeError(f"mb200_host build failed:\n{p.stdout}\n{p.stderr}")
    return LIB


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", "-v", action="store_true")
    args = ap.parse_args(argv)
    print(build(force=args.force, verbose=args.verbose))


if __name__ == "__main__":
    main()
