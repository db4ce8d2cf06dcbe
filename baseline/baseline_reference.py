"""Reference arm of bench.py (see reference_arm.py for the implementation)."""
from reference_arm import run  # noqa: F401
