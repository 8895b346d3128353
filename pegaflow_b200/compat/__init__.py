"""Drop-in support for the reference's own Python package.

``install(package_dir)`` puts ``pegaflow.py`` (this directory's stand-in for
the compiled ``pegaflow.pegaflow`` extension) into an installed copy of the
reference's ``pegaflow`` package. A compiled extension found there is renamed
aside (``*.so.disabled``), because Python's import system prefers an extension
module over a source file of the same name.
"""

from __future__ import annotations

import shutil
from pathlib import Path

SHIM = Path(__file__).resolve().parent / "pegaflow.py"


def install(package_dir: str | Path) -> Path:
    """Install the stand-in into the reference package at `package_dir` (the
    directory holding its ``__init__.py``); returns the written file."""
    pkg = Path(package_dir)
    if not (pkg / "__init__.py").exists():
        raise FileNotFoundError(f"{pkg} is not a Python package directory")
    for ext in pkg.glob("pegaflow.*.so"):
        ext.rename(ext.with_name(ext.name + ".disabled"))
    target = pkg / "pegaflow.py"
    if target.is_symlink():
        target.unlink()
    shutil.copyfile(SHIM, target)
    return target
