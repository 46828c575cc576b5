"""Install recipe for the reference package under ``baseline/_ref``.

The reference (``qtts``, pure Python: its GPU kernels are Triton) is installed
with the offline wheelhouse and no dependency resolution, from a copy of its
source tree (the setuptools build writes ``build/`` and ``*.egg-info`` beside
the sources, and the original tree is read-only)::

    python -m pip install --no-index --no-build-isolation --no-deps \
        --find-links /opt/wheelhouse --target baseline/_ref <copy of the reference>

``baseline/_ref`` is git-ignored but travels with the repository snapshot to
the GPU box, so the benchmark and the GPU tests find it there.

``python -m baseline.install [SOURCE]`` runs the recipe; ``__graft_entry__.build()``
calls :func:`install` when the reference source is present and ``_ref`` is not.
"""

from __future__ import annotations

import shutil
import subprocess
import sys
import tempfile
from pathlib import Path

HERE = Path(__file__).resolve().parent
TARGET = HERE / "_ref"
DEFAULT_SOURCE = Path("/root/reference")
WHEELHOUSE = Path("/opt/wheelhouse")


def installed() -> bool:
    return (TARGET / "qtts" / "quant" / "kernels.py").is_file()


def install(source: Path | str = DEFAULT_SOURCE, force: bool = False) -> bool:
    """Install the reference into ``baseline/_ref``. Returns False when ``source``
    does not exist (e.g. on the GPU box, which only uses the installed copy)."""
    source = Path(source)
    if installed() and not force:
        return True
    if not (source / "pyproject.toml").is_file():
        return False
    with tempfile.TemporaryDirectory(prefix="qtts_ref_src_") as tmp:
        copy = Path(tmp) / "src"
        shutil.copytree(source, copy, ignore=shutil.ignore_patterns(".git", "__pycache__"))
        if TARGET.exists():
            shutil.rmtree(TARGET)
        cmd = [sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation", "--no-deps",
               "--quiet", "--target", str(TARGET)]
        if WHEELHOUSE.is_dir():
            cmd += ["--find-links", str(WHEELHOUSE)]
        cmd.append(str(copy))
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"reference install failed ({proc.returncode}):\n{proc.stdout}\n{proc.stderr}")
    return installed()


if __name__ == "__main__":
    src = sys.argv[1] if len(sys.argv) > 1 else DEFAULT_SOURCE
    ok = install(src, force="--force" in sys.argv)
    print(f"reference installed at {TARGET}" if ok else f"no reference source at {src}")
