"""Build of the sm_100a shared library behind the C ABI.

``build()`` compiles every ``csrc/*.cu`` with nvcc for ``sm_100a`` into
``agentkv_b200/libagentkv_b200.so`` (in-tree, so it travels with the source
tree).  The CUDA runtime is linked statically: the library needs no CUDA
library at load time and exports only the ``akv_*`` C symbols declared in
``include/agentkv_b200.h``.  It also compiles ``csrc/akv_pyhost.c``, a small
CPython extension (``agentkv_b200._akv_pyhost``) that reads a batch's token
array addresses for the host-side packing of lookups.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sysconfig
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC_DIR = PKG_DIR / "csrc"
INCLUDE_DIR = REPO_DIR / "include"
LIB_NAME = "libagentkv_b200.so"
LIB_PATH = PKG_DIR / LIB_NAME
HOST_EXT_SRC = CSRC_DIR / "akv_pyhost.c"
HOST_EXT_PATH = PKG_DIR / ("_akv_pyhost" + (sysconfig.get_config_var("EXT_SUFFIX") or ".so"))

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC,-fvisibility=hidden,-pthread",
    "-lpthread",
    "-cudart",
    "static",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; the agentkv_b200 CUDA library cannot be built")


def sources() -> list[Path]:
    return sorted(CSRC_DIR.glob("*.cu"))


def _stale() -> bool:
    if not LIB_PATH.exists():
        return True
    t = LIB_PATH.stat().st_mtime
    deps = sources() + sorted(CSRC_DIR.glob("*.cuh")) + sorted(INCLUDE_DIR.glob("*.h"))
    return any(p.stat().st_mtime > t for p in deps)


def build_host_ext(force: bool = False, verbose: bool = False) -> Path:
    """Compile the CPython host helper if its source is newer than it."""
    if not force and HOST_EXT_PATH.exists() and HOST_EXT_PATH.stat().st_mtime >= HOST_EXT_SRC.stat().st_mtime:
        return HOST_EXT_PATH
    cc = os.environ.get("CC") or shutil.which("gcc") or shutil.which("cc")
    if not cc:
        raise RuntimeError("no C compiler found; the agentkv_b200 host helper cannot be built")
    tmp = HOST_EXT_PATH.with_name(HOST_EXT_PATH.name + ".tmp")
    cmd = [cc, "-O2", "-shared", "-fPIC", "-fvisibility=hidden", f"-I{sysconfig.get_paths()['include']}",
           str(HOST_EXT_SRC), "-o", str(tmp)]
    if verbose:
        print(" ".join(cmd))
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"{cc} failed ({proc.returncode}):\n{proc.stdout}\n{proc.stderr}")
    os.replace(tmp, HOST_EXT_PATH)
    return HOST_EXT_PATH


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile the library (and the host helper) if any source is newer than
    it; return the library's path."""
    build_host_ext(force, verbose)
    if not force and not _stale():
        return LIB_PATH
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [_nvcc(), *ARCH_FLAGS, *NVCC_FLAGS, f"-I{INCLUDE_DIR}", "-shared", "-o", str(tmp)]
    cmd += [str(p) for p in sources()]
    if verbose:
        print(" ".join(cmd))
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed ({proc.returncode}):\n{proc.stdout}\n{proc.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force=True, verbose=True))
