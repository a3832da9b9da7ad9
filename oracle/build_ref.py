"""Builds the reference's own C++ paged-attention op into ``oracle/_ref/``.

Test infrastructure: the op is compiled from ``csrc/paged_attention.cpp`` where
it lies in the reference checkout (read-only; nothing is copied), with torch's
extension builder and the reference's own flag (-O3, setup.py:8-12), into the
git-ignored ``oracle/_ref/``.  The built module travels with the repository to
machines without the checkout, where ``oracle.load_reference_op()`` imports it
directly.  The reference's own build system (setup.py) is not run.

    python oracle/build_ref.py <reference checkout>   (or BS_REFERENCE_DIR)
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"


def reference_root(explicit: str | Path | None = None) -> Path | None:
    """The reference checkout: the given path, else BS_REFERENCE_DIR, else none."""
    found = explicit or os.environ.get("BS_REFERENCE_DIR")
    return Path(found) if found else None


def build(root: str | Path | None = None) -> Path | None:
    """Builds the op from the checkout at `root` (or BS_REFERENCE_DIR); returns
    the module's path, or None without a checkout."""
    root = reference_root(root)
    if root is None:
        return None
    source = root / "csrc" / "paged_attention.cpp"
    if not source.exists():
        return None
    existing = sorted(OUT.glob("paged_attention_cpp*.so"))
    if existing and existing[0].stat().st_mtime >= source.stat().st_mtime:
        return existing[0]
    from torch.utils.cpp_extension import load

    OUT.mkdir(exist_ok=True)
    load(
        name="paged_attention_cpp",
        sources=[str(source)],
        extra_cflags=["-O3"],
        build_directory=str(OUT),
        verbose=False,
    )
    built = sorted(OUT.glob("paged_attention_cpp*.so"))
    return built[0] if built else None


if __name__ == "__main__":
    print(build(sys.argv[1] if len(sys.argv) > 1 else None))
