"""Build libmgc_cuda.so with nvcc for sm_100a, in tree.

The counterpart of the reference's C build driver (``codegen/build.py:129-209``): the compiler is
``$MGC_NVCC``, else ``nvcc`` on the PATH, else ``/usr/local/cuda/bin/nvcc``; the library is
rebuilt only when the hash of the sources and flags changes (the key is stored next to the
library), and written atomically. Unlike the C backend there is one library for every model:
a model is data (a launch list and a weights blob), not generated source.
"""

from __future__ import annotations

import hashlib
import os
import shutil
import subprocess
from pathlib import Path

from mgc_cuda import _reference  # noqa: F401
from ml_graph_compiler.errors import CodegenError

PACKAGE_DIR = Path(__file__).resolve().parent
SRC_DIR = PACKAGE_DIR.parent / "csrc"
INCLUDE_DIR = PACKAGE_DIR.parents[1] / "include"
LIB_DIR = PACKAGE_DIR / "lib"
LIB_NAME = "libmgc_cuda.so"
ARCH = os.environ.get("MGC_CUDA_ARCH", "sm_100a")


def find_nvcc() -> str:
    for cand in (os.environ.get("MGC_NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise CodegenError("nvcc not found (set MGC_NVCC)")


def nvcc_flags() -> list[str]:
    arch = ARCH.replace("sm_", "")
    return [
        "-O3",
        "-std=c++17",
        "-lineinfo",
        f"-gencode=arch=compute_{arch},code=sm_{arch}",
        "-Xcompiler=-fPIC,-O3,-Wall,-Wno-unused-function",
        "-shared",
        "--expt-relaxed-constexpr",
        f"-I{INCLUDE_DIR}",
        f"-I{SRC_DIR}",
    ]


def sources() -> list[Path]:
    return sorted([*SRC_DIR.glob("*.cu"), *SRC_DIR.glob("*.cuh"), *INCLUDE_DIR.glob("*.h")])


def source_key(flags: list[str]) -> str:
    h = hashlib.sha256()
    for path in sources():
        h.update(path.name.encode())
        h.update(path.read_bytes())
    for f in flags:
        h.update(f.encode())
    return h.hexdigest()[:20]


def library_path() -> Path:
    return LIB_DIR / LIB_NAME


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile the library if the sources changed; return its path."""
    flags = nvcc_flags()
    key = source_key(flags)
    lib = library_path()
    stamp = lib.with_suffix(".key")
    if not force and lib.exists() and stamp.exists() and stamp.read_text().strip() == key:
        return lib
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    tmp = lib.with_name(f"{LIB_NAME}.tmp{os.getpid()}")
    cmd = [find_nvcc(), *flags, str(SRC_DIR / "mgc_cuda.cu"), "-o", str(tmp)]
    if verbose:
        print(" ".join(cmd))
    proc = subprocess.run(cmd, capture_output=True, text=True, check=False)
    if proc.returncode != 0:
        raise CodegenError(f"nvcc failed:\n{' '.join(cmd)}\n{proc.stderr[-6000:]}")
    if verbose and proc.stderr:
        print(proc.stderr[-6000:])
    tmp.replace(lib)
    stamp.write_text(key + "\n")
    return lib


if __name__ == "__main__":
    print(build(force=True, verbose=True))
