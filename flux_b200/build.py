"""Build ``libfluxb200.so`` (sm_100a) from ``flux_b200/csrc`` with nvcc.

    python -m flux_b200.build [--verbose]

Each ``.cu`` compiles to an object under ``flux_b200/_build`` (rebuilt when the
source, a header or the flags change) and the objects link into
``flux_b200/_lib/libfluxb200.so`` with the CUDA runtime linked statically.
nvcc cross-compiles, so this runs on a host without a GPU.  Then
``csrc/torch_classes.cpp`` (the ``torch.classes.flux`` runtime classes over
the C ABI) compiles with the host compiler against PyTorch's headers into
``flux_b200/_lib/libfluxb200_torch.so``.
"""

from __future__ import annotations

import argparse
import hashlib
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
ROOT = PACKAGE.parent
CSRC = PACKAGE / "csrc"
BUILD = PACKAGE / "_build"
LIB_DIR = PACKAGE / "_lib"
LIBRARY = LIB_DIR / "libfluxb200.so"
TORCH_LIBRARY = LIB_DIR / "libfluxb200_torch.so"
TORCH_SOURCE = CSRC / "torch_classes.cpp"
INCLUDE = ROOT / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-I", str(INCLUDE), "-I", str(CSRC),
]


def nvcc() -> str:
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(found).exists():
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build flux_b200")
    return found


def _headers() -> list[Path]:
    return sorted([*CSRC.glob("*.cuh"), *CSRC.glob("*.h"), *INCLUDE.glob("*.h")])


def _stamp(source: Path, flags: list[str]) -> str:
    h = hashlib.sha256()
    h.update(" ".join(flags).encode())
    for path in [source, *_headers()]:
        h.update(path.read_bytes())
    return h.hexdigest()


def _compile(source: Path, flags: list[str], verbose: bool) -> Path:
    obj = BUILD / (source.stem + ".o")
    stamp = BUILD / (source.stem + ".stamp")
    digest = _stamp(source, flags)
    if obj.exists() and stamp.exists() and stamp.read_text() == digest:
        return obj
    cmd = [nvcc(), *flags, "-c", str(source), "-o", str(obj)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"nvcc failed for {source.name}:\n{result.stdout}\n{result.stderr}")
    if verbose and result.stderr:
        print(result.stderr, flush=True)
    stamp.write_text(digest)
    return obj


def build(verbose: bool = False, jobs: int | None = None) -> Path:
    """Compile and link the library; returns its path."""
    BUILD.mkdir(exist_ok=True)
    LIB_DIR.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    jobs = jobs or min(len(sources), os.cpu_count() or 1)
    with ThreadPoolExecutor(max_workers=jobs) as pool:
        objects = list(pool.map(lambda s: _compile(s, NVCC_FLAGS, verbose), sources))
    newest = max(o.stat().st_mtime for o in objects)
    if not LIBRARY.exists() or LIBRARY.stat().st_mtime < newest:
        tmp = LIBRARY.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objects)]
        result = subprocess.run(cmd, capture_output=True, text=True)
        if result.returncode != 0:
            raise RuntimeError(f"link failed:\n{result.stdout}\n{result.stderr}")
        os.replace(tmp, LIBRARY)
    return LIBRARY


def _torch_flags() -> list[str]:
    import torch
    import torch.utils.cpp_extension as ext
    includes = ext.include_paths(device_type="cuda")
    libraries = ext.library_paths(device_type="cuda")
    torch_lib = str(Path(torch.__file__).resolve().parent / "lib")
    return ["-O2", "-std=c++17", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}",
            *(f"-I{p}" for p in includes), f"-I{INCLUDE}", f"-I{CSRC}",
            *(f"-L{p}" for p in libraries), f"-Wl,-rpath,{torch_lib}", "-Wl,-rpath,$ORIGIN"]


def build_torch_classes(verbose: bool = False) -> Path:
    """The ``torch.classes.flux`` library (links ``libfluxb200.so`` and libtorch)."""
    library = build(verbose=verbose)
    flags = _torch_flags()
    stamp = BUILD / "torch_classes.stamp"
    h = hashlib.sha256()
    h.update(" ".join(flags).encode())
    for path in [TORCH_SOURCE, INCLUDE / "flux_b200.h"]:
        h.update(path.read_bytes())
    digest = h.hexdigest()
    if (TORCH_LIBRARY.exists() and stamp.exists() and stamp.read_text() == digest
            and TORCH_LIBRARY.stat().st_mtime >= library.stat().st_mtime):
        return TORCH_LIBRARY
    tmp = TORCH_LIBRARY.with_suffix(".so.tmp")
    cmd = [os.environ.get("CXX", "g++"), *flags, str(TORCH_SOURCE), "-o", str(tmp), f"-L{LIB_DIR}", "-lfluxb200",
           "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda"]
    if verbose:
        print(" ".join(cmd), flush=True)
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"building the torch classes failed:\n{result.stdout}\n{result.stderr}")
    os.replace(tmp, TORCH_LIBRARY)
    stamp.write_text(digest)
    return TORCH_LIBRARY


def main(argv: list[str] | None = None) -> int:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--verbose", action="store_true", help="print nvcc commands and ptxas resource usage")
    parser.add_argument("--jobs", type=int, default=None)
    args = parser.parse_args(argv)
    path = build(verbose=args.verbose, jobs=args.jobs)
    print(path)
    print(build_torch_classes(verbose=args.verbose))
    return 0


if __name__ == "__main__":
    sys.exit(main())
