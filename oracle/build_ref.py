"""Builds the REFERENCE's own CUDA operator library from its sources, for sm_100a.

TEST INFRASTRUCTURE ONLY.  The reference's csrc/register.cpp, csrc/gdn_decode.cu and
csrc/state_io.cu (with include/lightdelta/ops.h) are compiled where they lie, unmodified, into
oracle/_ref/_C.so -- the same torch.library `lightdelta` namespace the product registers, so it
must be loaded in a process of its own.  The GPU tests use it as a second, independent oracle
(the reference kernel itself at its HV=48 geometry) and as the kernel to compare against.
Nothing is copied from the reference tree; nothing is written outside oracle/_ref/.

It also builds oracle/_ref/libref_harness.so from oracle/ref_geometry_harness.cu, which includes
the reference's csrc/gdn_decode.cu unmodified and launches its kernel template at value-head ratio
2 or 3 through one C function (the stock launcher only runs ratio 3, HV=48), so the reference
kernel can run at the BASELINE geometry (H=16, HV=32).  It registers no torch operators, so it
can share a process with lightdelta_b200.

And it byte-compiles the reference's torch decode path -- python/lightdelta/__init__.py and
python/lightdelta/reference/{__init__,gdn}.py, unmodified -- into oracle/_ref/torch_path/, one
"<module name>.bytecode" file each (the .pyc format under another name, loaded by
oracle/ref_torch.py), so that the reference's own CPU implementation can be timed on a host where the
reference tree is absent.

Run here (where the reference sources exist):  python oracle/build_ref.py [--reference DIR]
"""

from __future__ import annotations

import argparse
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT_DIR = HERE / "_ref"
OUT = OUT_DIR / "_C.so"
# The reference checkout sits beside this repository ("reference" next to the repo's directory);
# LIGHTDELTA_REFERENCE overrides it.
DEFAULT_REFERENCE = Path(os.environ.get("LIGHTDELTA_REFERENCE", HERE.parent.parent / "reference"))
SOURCES = ("csrc/register.cpp", "csrc/gdn_decode.cu", "csrc/state_io.cu")


def _torch_flags():
    import torch
    from torch.utils import cpp_extension

    includes = cpp_extension.include_paths() + ["/usr/local/cuda/include"]
    lib = str(Path(torch.__file__).resolve().parent / "lib")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    return includes, lib, abi


def build(reference: Path = DEFAULT_REFERENCE, force: bool = False) -> Path:
    sources = [reference / s for s in SOURCES]
    missing = [str(s) for s in sources if not s.exists()]
    if missing:
        raise FileNotFoundError(f"reference sources not found: {missing}")
    if OUT.exists() and not force and all(s.stat().st_mtime <= OUT.stat().st_mtime for s in sources):
        return OUT
    OUT_DIR.mkdir(parents=True, exist_ok=True)
    includes, lib, abi = _torch_flags()
    inc = [f"-I{p}" for p in includes] + [f"-I{reference / 'include'}"]
    defs = [f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_EXTENSION_NAME=_C"]
    objs = []
    for src in sources:
        obj = OUT_DIR / (src.name + ".o")
        if src.suffix == ".cu":
            cmd = ["/usr/local/cuda/bin/nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17",
                   "--expt-relaxed-constexpr", "-lineinfo", "-Xcompiler", "-fPIC", *defs, *inc, "-c", str(src),
                   "-o", str(obj)]
        else:
            cmd = [os.environ.get("CXX", "g++"), "-O3", "-std=c++17", "-fPIC", *defs, *inc, "-c", str(src), "-o",
                   str(obj)]
        subprocess.run(cmd, check=True)
        objs.append(str(obj))
    tmp = OUT.with_suffix(".tmp.so")
    subprocess.run(["/usr/local/cuda/bin/nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-shared", *objs,
                    "-o", str(tmp), f"-L{lib}", "-lc10", "-lc10_cuda", "-ltorch_cpu", "-ltorch",
                    f"-Xlinker=-rpath,{lib}"], check=True)
    os.replace(tmp, OUT)
    for obj in objs:
        Path(obj).unlink(missing_ok=True)
    return OUT


HARNESS_SRC = HERE / "ref_geometry_harness.cu"
HARNESS = OUT_DIR / "libref_harness.so"


def build_harness(reference: Path = DEFAULT_REFERENCE, force: bool = False) -> Path:
    kernel = reference / "csrc" / "gdn_decode.cu"
    if not kernel.exists():
        raise FileNotFoundError(f"reference kernel not found: {kernel}")
    deps = [kernel, HARNESS_SRC, reference / "include" / "lightdelta" / "ops.h"]
    if HARNESS.exists() and not force and all(d.stat().st_mtime <= HARNESS.stat().st_mtime for d in deps):
        return HARNESS
    OUT_DIR.mkdir(parents=True, exist_ok=True)
    includes, lib, abi = _torch_flags()
    tmp = HARNESS.with_suffix(".tmp.so")
    cmd = ["/usr/local/cuda/bin/nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17",
           "--expt-relaxed-constexpr", "-lineinfo", "-shared", "-Xcompiler", "-fPIC",
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}", *[f"-I{p}" for p in includes], f"-I{reference}",
           f"-I{reference / 'include'}", str(HARNESS_SRC), "-o", str(tmp), f"-L{lib}", "-lc10", "-lc10_cuda",
           "-ltorch_cpu", "-ltorch", f"-Xlinker=-rpath,{lib}"]
    subprocess.run(cmd, check=True)
    os.replace(tmp, HARNESS)
    return HARNESS


TORCH_PATH_DIR = OUT_DIR / "torch_path"
# module name -> source under the reference's python/ directory, in the order they are loaded
TORCH_PATH_MODULES = {
    "lightdelta": "lightdelta/__init__.py",
    "lightdelta.reference.gdn": "lightdelta/reference/gdn.py",
    "lightdelta.reference": "lightdelta/reference/__init__.py",
}


def build_torch_path(reference: Path = DEFAULT_REFERENCE, force: bool = False) -> Path:
    """Compiles the reference's torch path to bytecode: the package marker and post_conv_gdn, which
    import nothing of the reference beyond each other."""
    import py_compile

    TORCH_PATH_DIR.mkdir(parents=True, exist_ok=True)
    for name, relative in TORCH_PATH_MODULES.items():
        src = reference / "python" / relative
        if not src.exists():
            raise FileNotFoundError(f"reference module not found: {src}")
        dst = TORCH_PATH_DIR / f"{name}.bytecode"
        if dst.exists() and not force and src.stat().st_mtime <= dst.stat().st_mtime:
            continue
        py_compile.compile(str(src), cfile=str(dst), doraise=True,
                           invalidation_mode=py_compile.PycInvalidationMode.UNCHECKED_HASH)
    return TORCH_PATH_DIR


def build_if_available() -> Path | None:
    """Builds oracle/_ref/_C.so (and the harness and the torch path's bytecode) when the reference
    sources are present (this container); on the GPU box the prebuilt files are used as shipped."""
    if not DEFAULT_REFERENCE.exists():
        return OUT if OUT.exists() else None
    build_harness(DEFAULT_REFERENCE)
    build_torch_path(DEFAULT_REFERENCE)
    return build(DEFAULT_REFERENCE)


def main() -> int:
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--reference", type=Path, default=DEFAULT_REFERENCE)
    parser.add_argument("--force", action="store_true")
    args = parser.parse_args()
    print(build(args.reference, args.force))
    print(build_harness(args.reference, args.force))
    print(build_torch_path(args.reference, args.force))
    return 0


if __name__ == "__main__":
    sys.exit(main())
