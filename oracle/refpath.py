"""Location of the reference checkout -- test infrastructure only.

The checkers that are built from the reference's own sources (``oracle/_ref``) and
the scripts that generate golden fixtures need the reference project's sources.
Their location is taken from the environment variable ``DELTAGRID_REF``; when it
is unset, from the one-line file ``oracle/reference.cfg``, a path relative to the
repository root.  Nothing on the product path, in the GPU tests, in ``smoke()`` or
in ``bench.py`` reads it: the checkers travel prebuilt in ``oracle/_ref/``.

    python oracle/refpath.py      # prints the resolved directory, or exits 1
"""
from __future__ import annotations

import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CFG = os.path.join(HERE, "reference.cfg")


def reference_root(required: bool = True) -> str | None:
    """The reference checkout directory, or None (``required=False``) when it cannot be found."""
    path = os.environ.get("DELTAGRID_REF")
    how = "DELTAGRID_REF"
    if not path and os.path.exists(CFG):
        with open(CFG) as f:
            rel = f.read().strip()
        if rel:
            path = os.path.normpath(os.path.join(REPO, rel))
            how = f"oracle/reference.cfg ({rel!r} relative to the repository root)"
    if path and os.path.isdir(os.path.join(path, "src")):
        return path
    if required:
        raise RuntimeError(
            "reference checkout not found: set DELTAGRID_REF to the reference project's root "
            f"(tried {how}: {path!r})" if path else
            "reference checkout not found: set DELTAGRID_REF to the reference project's root")
    return None


if __name__ == "__main__":
    root = reference_root(required=False)
    if root is None:
        sys.exit(1)
    print(root)
