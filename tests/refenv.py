"""Test-side name of oracle/reference_gpu.py (the unmodified reference next to this
library in one process)."""
from oracle.reference_gpu import EXAMPLES, STAGED, Reference, missing  # noqa: F401
