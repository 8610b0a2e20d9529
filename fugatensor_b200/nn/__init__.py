"""Neural-network functionals built from Fuga primitives."""
from . import functional  # noqa: F401
