"""``mlx.nn`` subset on numpy (see package docstring)."""
import numpy as np


class Module:
    def __init__(self, *a, **k):
        pass

    def __call__(self, *args, **kw):
        return self.forward(*args, **kw)


def silu(x):
    return x / (1.0 + np.exp(-x))
