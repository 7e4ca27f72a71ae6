"""Torch-CPU ``mlx`` stand-in: test infrastructure for golden-fixture generation only."""
from . import core, nn  # noqa: F401
