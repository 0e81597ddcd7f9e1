"""Build libfgw_mha.so in-tree with nvcc for sm_100a.

Each ``csrc/*.cu`` compiles to an object under ``_build/`` in parallel; the objects link into
``fgw_b200/_lib/libfgw_mha.so`` with the CUDA runtime linked statically, so the library only
needs the NVIDIA driver at run time. Re-running is incremental (objects newer than their
sources and headers are kept).

    python -m fgw_b200.build [--force] [--jobs N]
"""
import argparse
import concurrent.futures
import os
import pathlib
import shutil
import subprocess
import sys

PACKAGE = pathlib.Path(__file__).resolve().parent
ROOT = PACKAGE.parent
CSRC = PACKAGE / "csrc"
INCLUDE = ROOT / "include"
BUILD = ROOT / "_build"
LIB_DIR = PACKAGE / "_lib"
LIB = LIB_DIR / "libfgw_mha.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
# Host code keeps separate multiplies and adds (no fused multiply-add contraction): the host split choice
# (fgw_split_choice.cu) must round like its Python restatement to make the same picks.
CFLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
          "--expt-relaxed-constexpr", "-DNDEBUG", "-Xcompiler", "-ffp-contract=off", f"-I{INCLUDE}", f"-I{CSRC}"]


def nvcc():
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(found):
        raise RuntimeError("nvcc not found; the CUDA 12.9 toolkit is required to build libfgw_mha.so")
    return found


def _stale(obj, src, headers):
    if not obj.exists():
        return True
    stamp = obj.stat().st_mtime
    return any(p.stat().st_mtime > stamp for p in [src, *headers])


def _compile(src, obj, extra):
    cmd = [nvcc(), *ARCH, *CFLAGS, *extra, "-c", str(src), "-o", str(obj)]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{proc.stdout}\n{proc.stderr}")
    return proc.stderr


def build(force=False, jobs=None, verbose_ptxas=False):
    """Compile every kernel translation unit and link the shared library; returns its path."""
    BUILD.mkdir(exist_ok=True)
    LIB_DIR.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    headers = sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))
    extra = ["-Xptxas", "-v"] if verbose_ptxas else []
    objects = [BUILD / (s.stem + ".o") for s in sources]
    todo = [(s, o) for s, o in zip(sources, objects) if force or verbose_ptxas or _stale(o, s, headers)]
    logs = {}
    if todo:
        workers = jobs or min(len(todo), os.cpu_count() or 4)
        with concurrent.futures.ThreadPoolExecutor(workers) as pool:
            futures = {pool.submit(_compile, s, o, extra): s for s, o in todo}
            for fut in concurrent.futures.as_completed(futures):
                logs[futures[fut].name] = fut.result()
    if todo or not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objects):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objects)]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"link failed:\n{proc.stdout}\n{proc.stderr}")
        os.replace(tmp, LIB)
    if verbose_ptxas:
        for name, text in sorted(logs.items()):
            print(f"== {name}\n{text}")
    return LIB


def main(argv=None):
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--jobs", type=int, default=None)
    parser.add_argument("--ptxas", action="store_true", help="print -Xptxas -v register/smem usage")
    args = parser.parse_args(argv)
    path = build(force=args.force, jobs=args.jobs, verbose_ptxas=args.ptxas)
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
