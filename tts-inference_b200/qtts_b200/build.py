"""Build recipe for the sm_100a shared library behind the C ABI.

``python -m qtts_b200.build`` (or ``__graft_entry__.build()``) compiles every
``csrc/*.cu`` with nvcc for ``sm_100a`` only and links them into
``qtts_b200/lib/libqtts_b200.so``. The library links the CUDA runtime
statically and reaches the driver through ``cudaGetDriverEntryPoint``, so it
loads on a machine without a GPU (for the symbol checks) and carries no
dependency on torch.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
SRC_DIR = PKG_DIR.parent / "csrc"
REPO_DIR = PKG_DIR.parent.parent
INCLUDE_DIR = REPO_DIR / "include"
LIB_DIR = PKG_DIR / "lib"
LIB_PATH = LIB_DIR / "libqtts_b200.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-rdc=true",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
]


def nvcc_path() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    candidate = Path(cuda_home) / "bin" / "nvcc"
    if candidate.exists():
        return str(candidate)
    found = shutil.which("nvcc")
    if found is None:
        raise RuntimeError("nvcc not found (set CUDA_HOME)")
    return found


def sources() -> list[Path]:
    return sorted(SRC_DIR.glob("*.cu"))


def _stale() -> bool:
    if not LIB_PATH.exists():
        return True
    built = LIB_PATH.stat().st_mtime
    deps = list(SRC_DIR.glob("*")) + list(INCLUDE_DIR.glob("*.h"))
    return any(p.stat().st_mtime > built for p in deps)


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed ({proc.returncode}):\n{proc.stdout}\n{proc.stderr}")
    if verbose and (proc.stdout or proc.stderr):
        print(proc.stdout + proc.stderr, file=sys.stderr)


def build(force: bool = False, verbose: bool = False, extra_flags: list[str] | None = None) -> Path:
    """Compile the library if any source is newer than it. Returns its path.

    Each source compiles to a relocatable object in parallel (``_build/``, one
    nvcc per file), then one nvcc call device-links and links them into the
    shared library."""
    if not force and not _stale():
        return LIB_PATH
    from concurrent.futures import ThreadPoolExecutor

    LIB_DIR.mkdir(parents=True, exist_ok=True)
    obj_dir = PKG_DIR.parent / "_build"
    obj_dir.mkdir(exist_ok=True)
    flags = ARCH_FLAGS + NVCC_FLAGS + (extra_flags or []) + ["-I", str(INCLUDE_DIR), "-I", str(SRC_DIR)]
    srcs = sources()
    objs = [obj_dir / (s.stem + ".o") for s in srcs]
    jobs = [[nvcc_path()] + flags + ["-c", str(s), "-o", str(o)] for s, o in zip(srcs, objs)]
    with ThreadPoolExecutor(max_workers=max(1, min(len(jobs), os.cpu_count() or 1))) as pool:
        for fut in [pool.submit(_run, cmd, verbose) for cmd in jobs]:
            fut.result()
    tmp = LIB_PATH.with_suffix(".so.tmp")
    _run([nvcc_path()] + ARCH_FLAGS + ["-shared", "-Xcompiler", "-fPIC", "-o", str(tmp)] + [str(o) for o in objs],
         verbose)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    force = "--force" in sys.argv
    path = build(force=force, verbose=True)
    print(path)
