"""Build the sm_100a shared library in-tree with nvcc (no JIT cache).

``python -m vllm_rlt_b200._build`` compiles every ``csrc/*.cu`` into
``vllm_rlt_b200/_lib/librlt_b200.so``. Objects are rebuilt only when their
source, a header or the flags changed. The library is plain C ABI
(``include/rlt_b200.h``) with the CUDA runtime linked statically.
"""

from __future__ import annotations

import concurrent.futures
import hashlib
import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
ROOT = PACKAGE.parent
CSRC = PACKAGE / "csrc"
OUT_DIR = PACKAGE / "_lib"
LIB_NAME = "librlt_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC",
    "-Xptxas",
    "-v",
    f"-I{ROOT / 'include'}",
    "--expt-relaxed-constexpr",
]


def nvcc() -> str:
    for candidate in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if candidate and Path(candidate).exists():
            return candidate
    raise RuntimeError("nvcc not found: the sm_100a library cannot be built")


def _digest(source: Path) -> str:
    h = hashlib.sha256()
    h.update(" ".join(ARCH + FLAGS).encode())
    h.update(source.read_bytes())
    for header in sorted(CSRC.glob("*.cuh")) + sorted((ROOT / "include").glob("*.h")):
        h.update(header.read_bytes())
    return h.hexdigest()[:16]


def _compile(source: Path, build_dir: Path, verbose: bool) -> Path:
    obj = build_dir / f"{source.stem}.{_digest(source)}.o"
    if obj.exists():
        return obj
    for stale in build_dir.glob(f"{source.stem}.*.o"):
        stale.unlink()
    cmd = [nvcc(), *ARCH, *FLAGS, "-c", str(source), "-o", str(obj)]
    result = subprocess.run(cmd, capture_output=True, text=True)
    log = build_dir / f"{source.stem}.ptxas.log"
    log.write_text(result.stdout + result.stderr)
    if result.returncode != 0:
        raise RuntimeError(f"nvcc failed for {source.name}:\n{result.stderr[-6000:]}")
    if verbose:
        print(f"compiled {source.name}", file=sys.stderr)
    return obj


def build(verbose: bool = False) -> Path:
    """Compile and link; return the path of the shared library."""
    build_dir = PACKAGE / "_build"
    build_dir.mkdir(exist_ok=True)
    OUT_DIR.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    workers = min(len(sources), os.cpu_count() or 1)
    with concurrent.futures.ThreadPoolExecutor(workers) as pool:
        objects = list(pool.map(lambda s: _compile(s, build_dir, verbose), sources))
    lib = OUT_DIR / LIB_NAME
    stamp = build_dir / "link.stamp"
    key = "\n".join(str(o) for o in objects)
    if lib.exists() and stamp.exists() and stamp.read_text() == key:
        return lib
    tmp = OUT_DIR / f".{LIB_NAME}.tmp"
    # Static cudart: the library depends only on the driver, and launches on
    # the caller's streams (torch's or anyone's) in the caller's primary context.
    cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objects)]
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"link failed:\n{result.stderr[-4000:]}")
    os.replace(tmp, lib)
    stamp.write_text(key)
    return lib


if __name__ == "__main__":
    print(build(verbose=True))
