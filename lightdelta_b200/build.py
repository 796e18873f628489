"""In-tree native build of lightdelta_b200 for sm_100a.

Produces, next to this file:
  liblightdelta_b200.so  the C-ABI library (kernels + entry points of include/lightdelta_b200.h),
                         built by nvcc with cudart linked statically, no torch dependency;
  _C.so                  the torch.library registration of the ``lightdelta`` namespace, a thin
                         g++-built layer over liblightdelta_b200.so (found through $ORIGIN).

Run ``python -m lightdelta_b200.build [--force]``.  Outputs are replaced atomically and only
rebuilt when a source or header is newer than the output.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
import tempfile
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
BUILD_DIR = ROOT / "_build" / "native"
CAPI_LIB = PKG / "liblightdelta_b200.so"
TORCH_LIB = PKG / "_C.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall"]

CAPI_SOURCES = ["gdn_decode.cu", "state_io.cu", "greedy_verify.cu", "conv_update.cu", "decode_noalloc.cu", "capi.cpp"]
CAPI_HEADERS = ["internal.h", "exports.map"]


def cuda_home() -> Path:
    return Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))


def nvcc() -> str:
    path = cuda_home() / "bin" / "nvcc"
    if path.exists():
        return str(path)
    found = shutil.which("nvcc")
    if not found:
        raise RuntimeError("nvcc not found: set CUDA_HOME to a CUDA 12.9+ toolkit")
    return found


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    mtime = target.stat().st_mtime
    return any(dep.stat().st_mtime > mtime for dep in deps)


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd), flush=True)
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"command failed ({result.returncode}): {' '.join(cmd)}\n{result.stdout}\n{result.stderr}")
    if verbose and (result.stdout or result.stderr):
        print(result.stdout + result.stderr, flush=True)


def _atomic_output(target: Path) -> Path:
    fd, tmp = tempfile.mkstemp(prefix=f".{target.name}.", suffix=".tmp", dir=target.parent)
    os.close(fd)
    return Path(tmp)


def build_capi(force: bool = False, verbose: bool = False) -> Path:
    sources = [CSRC / s for s in CAPI_SOURCES]
    deps = sources + [CSRC / h for h in CAPI_HEADERS] + [INCLUDE / "lightdelta_b200.h"]
    if not force and not _stale(CAPI_LIB, deps):
        return CAPI_LIB
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    objects = [BUILD_DIR / (s.stem + ".o") for s in sources]

    def compile_one(pair):
        src, obj = pair
        _run([nvcc(), *ARCH_FLAGS, *NVCC_FLAGS, f"-I{INCLUDE}", f"-I{CSRC}", "-c", str(src), "-o", str(obj)], verbose)

    with ThreadPoolExecutor(max_workers=len(sources)) as pool:
        list(pool.map(compile_one, zip(sources, objects)))
    tmp = _atomic_output(CAPI_LIB)
    try:
        _run([nvcc(), *ARCH_FLAGS, "-shared", "-Xlinker", f"-soname={CAPI_LIB.name}",
              "-Xlinker", f"--version-script={CSRC / 'exports.map'}", *map(str, objects),
              "-o", str(tmp)], verbose)
        os.replace(tmp, CAPI_LIB)
    finally:
        tmp.unlink(missing_ok=True)
    return CAPI_LIB


def _torch_paths() -> tuple[list[str], list[str], bool]:
    import torch
    from torch.utils import cpp_extension

    includes = cpp_extension.include_paths()
    includes.append(str(cuda_home() / "include"))
    libs = [str(Path(torch.__file__).resolve().parent / "lib")]
    return includes, libs, bool(torch._C._GLIBCXX_USE_CXX11_ABI)


def build_torch_ops(force: bool = False, verbose: bool = False) -> Path:
    source = CSRC / "torch_ops.cpp"
    deps = [source, INCLUDE / "lightdelta_b200.h", CAPI_LIB]
    if not force and not _stale(TORCH_LIB, deps):
        return TORCH_LIB
    includes, libs, cxx11 = _torch_paths()
    tmp = _atomic_output(TORCH_LIB)
    cmd = [
        os.environ.get("CXX", "g++"), "-O2", "-std=c++17", "-fPIC", "-shared", "-Wall",
        f"-D_GLIBCXX_USE_CXX11_ABI={int(cxx11)}",
        *[f"-I{p}" for p in includes], f"-I{INCLUDE}",
        str(source), "-o", str(tmp),
        f"-L{PKG}", f"-l:{CAPI_LIB.name}",
        *[f"-L{p}" for p in libs], "-lc10", "-lc10_cuda", "-ltorch_cpu", "-ltorch",
        "-Wl,-rpath,$ORIGIN", *[f"-Wl,-rpath,{p}" for p in libs],
    ]
    try:
        _run(cmd, verbose)
        os.replace(tmp, TORCH_LIB)
    finally:
        tmp.unlink(missing_ok=True)
    return TORCH_LIB


def build_all(force: bool = False, verbose: bool = False) -> list[Path]:
    return [build_capi(force, verbose), build_torch_ops(force, verbose)]


def main(argv: list[str] | None = None) -> int:
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--verbose", action="store_true")
    args = parser.parse_args(argv)
    for path in build_all(args.force, args.verbose):
        print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
