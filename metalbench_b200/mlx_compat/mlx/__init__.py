"""numpy stand-in for the subset of MLX that the hot-path hook files use.

MLX (the reference's CPU/GPU array library, ``mlx>=0.18.0``) exists only for
Apple Silicon. The harness puts this package's directory on ``sys.path`` as
``mlx`` when the real one cannot be imported, so the reference-style hooks under
``mlx/kernels/`` run unchanged on Linux: as the correctness reference of
``./bench`` and as the "MLX" timing leg (reported as ``mlx-compat(numpy)``).
Arrays are plain numpy arrays; each op follows MLX's published semantics for the
arguments the hooks pass. It never runs on the kernel path.
"""
from . import core, nn  # noqa: F401

__version__ = "0.0-numpy-compat"
