"""Import-compatibility module for ``from paged_decode.oracle import Layout``.

The reference keeps the plan's geometry type and metadata validator in
``paged_decode/oracle.py`` (oracle.py:11-47) next to its FP64 NumPy attention.
This package re-exports only the two plan-contract names from ``layout.py``;
it holds no attention math and no CPU fallback.  The FP64 checker used by the
tests lives outside the package.
"""
from .layout import Layout, validate_metadata

__all__ = ["Layout", "validate_metadata"]
