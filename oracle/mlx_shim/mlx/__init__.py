"""numpy stand-in for the subset of MLX that the hot-path reference hooks use.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``). Arrays are plain numpy
arrays; each op follows MLX's published semantics for the arguments the hooks
pass. It is put on ``sys.path`` only when the real ``mlx`` cannot be imported,
so that ``tests/golden/gen_golden.py`` can execute the reference's own hook
files and the harness can run its reference leg on Linux.
"""
from . import core, nn  # noqa: F401

__version__ = "0.0-numpy-shim"
