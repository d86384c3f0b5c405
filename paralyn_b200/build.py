"""Builds libparalyn_native.so in-tree: C++17 runtime + sm_100a CUDA kernels.

    python -m paralyn_b200.build [--force] [--jobs N]

Kernels are compiled ahead of time with nvcc for sm_100a only
(-gencode arch=compute_100a,code=sm_100a); the runtime links the CUDA runtime
statically, so the library needs only the NVIDIA driver at run time. Objects go
to paralyn_b200/_build/ and are rebuilt when a source or header is newer.
"""
import argparse
import concurrent.futures
import os
from pathlib import Path
import shutil
import subprocess
import sys

PACKAGE = Path(__file__).resolve().parent
ROOT = PACKAGE.parent
CSRC = PACKAGE / "csrc"
INCLUDE = ROOT / "include"
BUILD = PACKAGE / "_build"
LIBRARY = PACKAGE / "libparalyn_native.so"
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA_HOME / "bin" / "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CXX_FLAGS = ["-std=c++17", "-O2", "-fPIC", "-fvisibility=hidden", "-Wall", "-Wextra",
             "-Wno-unused-parameter"]
CUDA_FLAGS = ["-std=c++17", "-O3", "-lineinfo", *ARCH, "-Xcompiler", "-fPIC,-fvisibility=hidden",
              "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills"]


def _headers():
    return [p for p in list(CSRC.rglob("*.hpp")) + list(CSRC.rglob("*.cuh")) + list(INCLUDE.rglob("*.h"))]


def _stale(target, sources):
    if not target.exists():
        return True
    stamp = target.stat().st_mtime
    return any(s.stat().st_mtime > stamp for s in sources)


def _compile(source, obj, verbose):
    includes = [f"-I{INCLUDE}", f"-I{CSRC}", f"-I{CUDA_HOME / 'include'}"]
    if source.suffix == ".cu":
        command = [NVCC, *CUDA_FLAGS, *includes, "-c", str(source), "-o", str(obj)]
    else:
        command = ["g++", *CXX_FLAGS, *includes, "-c", str(source), "-o", str(obj)]
    if verbose:
        print(" ".join(command), flush=True)
    result = subprocess.run(command, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"compiling {source.name} failed:\n{result.stdout}{result.stderr}")
    return result.stderr


def build(force=False, jobs=None, verbose=False):
    """Compiles what changed and links the library; returns its path."""
    if not Path(NVCC).exists():
        raise RuntimeError(f"nvcc not found at {NVCC}; set CUDA_HOME")
    BUILD.mkdir(exist_ok=True)
    sources = sorted(CSRC.rglob("*.cpp")) + sorted(CSRC.rglob("*.cu"))
    headers = _headers()
    work = []
    objects = []
    for source in sources:
        obj = BUILD / (source.relative_to(CSRC).as_posix().replace("/", "__") + ".o")
        objects.append(obj)
        if force or _stale(obj, [source, *headers]):
            work.append((source, obj))
    warnings = []
    with concurrent.futures.ThreadPoolExecutor(max_workers=jobs or os.cpu_count() or 4) as pool:
        for text in pool.map(lambda item: _compile(*item, verbose), work):
            if text.strip():
                warnings.append(text)
    if force or work or _stale(LIBRARY, objects):
        exports = BUILD / "exports.map"
        exports.write_text("{ global: pr_*; local: *; };\n")
        command = [NVCC, *ARCH, "-shared", "-cudart", "static", "-o", str(LIBRARY),
                   *map(str, objects), "-ldl", "-lpthread", "-lrt",
                   f"-Xlinker=--version-script={exports}"]
        if verbose:
            print(" ".join(command), flush=True)
        result = subprocess.run(command, capture_output=True, text=True)
        if result.returncode != 0:
            raise RuntimeError(f"linking failed:\n{result.stdout}{result.stderr}")
    for text in warnings:
        print(text, file=sys.stderr)
    from . import prk
    prk.write_operators(PACKAGE / "data" / "operators.prk")
    return LIBRARY


def clean():
    shutil.rmtree(BUILD, ignore_errors=True)
    LIBRARY.unlink(missing_ok=True)


def main():
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--jobs", type=int)
    parser.add_argument("--verbose", action="store_true")
    args = parser.parse_args()
    print(build(args.force, args.jobs, args.verbose))


if __name__ == "__main__":
    main()
