"""``mlx.nn`` subset on numpy (see package docstring)."""
import numpy as np


class Module:
    def __init__(self, *a, **k):
        pass

    def __call__(self, *args, **kw):
        return self.forward(*args, **kw)


def silu(x):
    return x / (1.0 + np.exp(-x))


def gelu(x):
    """Exact GELU, x * Phi(x) = 0.5 x (1 + erf(x / sqrt(2))) (MLX nn.gelu)."""
    from scipy.special import erf
    return (0.5 * x * (1.0 + erf(x / np.sqrt(2.0)))).astype(np.asarray(x).dtype)


class RMSNorm(Module):
    """x * rsqrt(mean(x^2, -1) + eps) * weight, weight initialised to ones."""

    def __init__(self, dims, eps=1e-5):
        super().__init__()
        self.eps = eps
        self.weight = np.ones((dims,), dtype=np.float32)

    def forward(self, x):
        v = np.mean(x * x, axis=-1, keepdims=True, dtype=x.dtype)
        return x * (1.0 / np.sqrt(v + self.eps)).astype(x.dtype) * self.weight.astype(x.dtype)


class Linear(Module):
    """y = x @ weight.T (+ bias); weight (out, in) drawn U(-1/sqrt(in), 1/sqrt(in))."""

    def __init__(self, input_dims, output_dims, bias=True):
        super().__init__()
        k = 1.0 / np.sqrt(input_dims)
        rng = np.random.default_rng(0)
        self.weight = rng.uniform(-k, k, (output_dims, input_dims)).astype(np.float32)
        self.bias = rng.uniform(-k, k, (output_dims,)).astype(np.float32) if bias else None

    def forward(self, x):
        y = x @ self.weight.T
        return y + self.bias if self.bias is not None else y
