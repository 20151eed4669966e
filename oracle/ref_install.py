"""Install the reference (ravirajb/infercache) for the CPU baseline arm.

The reference is a flat Python package that imports itself as ``inference``
and ships no setup.py / pyproject.toml, so ``pip install --target baseline/_ref
<reference>`` refuses it ("Neither 'setup.py' nor 'pyproject.toml' found").
This recipe does what such an install would produce: the package's modules
under ``baseline/_ref/inference/``, unmodified.  ``baseline/_ref`` is
git-ignored and travels with the repository to the GPU machine.

    python oracle/ref_install.py [--src /path/to/reference]

CPU BASELINE INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).
"""
from __future__ import annotations

import argparse
import os
import shutil
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
DEST = ROOT / "baseline" / "_ref" / "inference"


def install(src: str) -> Path:
    srcp = Path(src)
    if not (srcp / "hierarchical_cache.py").exists():
        raise FileNotFoundError(f"{src} does not hold the reference package")
    if DEST.exists():
        shutil.rmtree(DEST)
    DEST.mkdir(parents=True)
    for f in sorted(srcp.iterdir()):
        if f.is_file() and f.suffix in (".py", ".md") or f.name == "LICENSE":
            shutil.copy2(f, DEST / f.name)
    return DEST


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--src", default=os.environ.get("INFERCACHE_REF", "/root/reference"))
    print(install(ap.parse_args().src))


if __name__ == "__main__":
    main()
