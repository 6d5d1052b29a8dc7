"""Install the reference implementation into ``baseline/_ref`` (git-ignored).

The reference checkout has no packaging metadata (no ``setup.py`` or
``pyproject.toml``), so ``pip install --target baseline/_ref`` cannot install
it. This recipe does what that install would: it copies the reference's
modules, unmodified, into ``baseline/_ref`` so that its stock Triton path
(``triton_impl.DDPM`` -> ``_triton_kernels``) can be timed on a B200 as the
"existing kernel" comparison of ``bench.py``. Only the copy under
``baseline/_ref`` travels to a GPU box; nothing of the reference is committed.

Usage: ``python baseline/install_reference.py [REFERENCE_DIR]`` (default: the
``DDPM_REFERENCE_DIR`` environment variable). Called by ``build()`` of
``__graft_entry__.py`` when the reference checkout is present.
"""

from __future__ import annotations

import os
import shutil
import sys
from pathlib import Path

MODULES = ("triton_impl.py", "_triton_kernels.py", "unfold_impl.py")
TARGET = Path(__file__).resolve().parent / "_ref"


def install(src: str | os.PathLike) -> Path | None:
    """Copy the reference modules from ``src`` into ``baseline/_ref``; returns
    the target, or ``None`` when ``src`` does not hold them."""
    src = Path(src)
    if not all((src / m).is_file() for m in MODULES):
        return None
    TARGET.mkdir(parents=True, exist_ok=True)
    for m in MODULES:
        shutil.copyfile(src / m, TARGET / m)
    return TARGET


def main(argv: list[str] | None = None) -> int:
    argv = sys.argv[1:] if argv is None else argv
    src = argv[0] if argv else os.environ.get("DDPM_REFERENCE_DIR")
    if not src:
        print("usage: install_reference.py REFERENCE_DIR", file=sys.stderr)
        return 2
    out = install(src)
    if out is None:
        print(f"{src} does not hold {', '.join(MODULES)}", file=sys.stderr)
        return 1
    print(out)
    return 0


if __name__ == "__main__":
    sys.exit(main())
