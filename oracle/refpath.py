"""Location of the reference checkout -- test infrastructure only.

The checkers that are built from the reference's own sources (``oracle/_ref``) and
the scripts that generate golden fixtures need the reference project's sources.
Their location is taken from the environment variable ``DELTAGRID_REF`` alone; when
it is unset they stop with an error that says so (``__graft_entry__.build()`` then
keeps the prebuilt checkers).  Nothing on the product path, in the GPU tests, in
``smoke()`` or in ``bench.py`` reads it: the checkers travel prebuilt in
``oracle/_ref/``.

    python oracle/refpath.py      # prints the resolved directory, or exits 1
"""
from __future__ import annotations

import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)


def reference_root(required: bool = True) -> str | None:
    """The reference checkout directory, or None (``required=False``) when it cannot be found."""
    path = os.environ.get("DELTAGRID_REF")
    if path and os.path.isdir(os.path.join(path, "src")):
        return path
    if required:
        raise RuntimeError(
            f"DELTAGRID_REF={path!r} is not a reference checkout (no src/ under it)" if path else
            "DELTAGRID_REF is unset: set it to the reference project's root")
    return None


if __name__ == "__main__":
    root = reference_root(required=False)
    if root is None:
        sys.exit(1)
    print(root)
