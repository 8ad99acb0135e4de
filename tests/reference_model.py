"""Test infrastructure: the reference's own Python package, loaded by
oracle/reference_pkg.py (installed from the reference sources into baseline/_ref)."""
from oracle.reference_pkg import REF_SITE, load_reference_package, use_backend  # noqa: F401
