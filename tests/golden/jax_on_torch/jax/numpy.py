"""``jax.numpy`` subset on torch (fixture generation only).

Semantics kept from JAX: ``take_along_axis`` normalises negative indices;
``einsum(..., preferred_element_type=float32)`` multiplies bfloat16 inputs
exactly and accumulates in float32; float64 inputs stay float64 (the
x64-enabled reading of a float32 preference as a minimum precision).
"""

import builtins

import torch

float32 = torch.float32
float64 = torch.float64
bfloat16 = torch.bfloat16
float16 = torch.float16
int32 = torch.int32
int64 = torch.int64
bool_ = torch.bool


def _dt(d):
    if d is None:
        return None
    if d is builtins.bool:
        return torch.bool
    if d is builtins.float:
        return torch.float64
    if d is builtins.int:
        return torch.int64
    return d


torch.Tensor.astype = lambda self, d: self.to(_dt(d))  # JAX array method


def dtype(d):
    return _dt(d)


def promote_types(a, b):
    return torch.promote_types(_dt(a), _dt(b))


def asarray(x, dtype=None):
    t = x if isinstance(x, torch.Tensor) else torch.as_tensor(x)
    return t.to(_dt(dtype)) if dtype is not None else t


def _t(x, like=None):
    if isinstance(x, torch.Tensor):
        return x
    return torch.as_tensor(x, dtype=like.dtype if like is not None else None)


def abs(x):
    return torch.abs(x)


def where(c, a, b):
    if not isinstance(a, torch.Tensor) and not isinstance(b, torch.Tensor):
        a = torch.as_tensor(a)
    return torch.where(c, a, b)


def mean(x, axis=None, keepdims=False):
    return x.mean() if axis is None else x.mean(dim=axis, keepdim=keepdims)


def sum(x, axis=None, keepdims=False):
    return x.sum() if axis is None else x.sum(dim=axis, keepdim=keepdims)


def max(x, axis=None, keepdims=False):
    return x.max() if axis is None else torch.amax(x, dim=axis, keepdim=keepdims)


def maximum(a, b):
    if not isinstance(a, torch.Tensor) and not isinstance(b, torch.Tensor):
        return builtins.max(a, b)
    if not isinstance(b, torch.Tensor):
        return torch.clamp(a, min=b)
    if not isinstance(a, torch.Tensor):
        return torch.clamp(b, min=a)
    return torch.maximum(a, b)


def minimum(a, b):
    if not isinstance(a, torch.Tensor) and not isinstance(b, torch.Tensor):
        return builtins.min(a, b)
    if not isinstance(b, torch.Tensor):
        return torch.clamp(a, max=b)
    if not isinstance(a, torch.Tensor):
        return torch.clamp(b, max=a)
    return torch.minimum(a, b)


def ones(shape, dtype=None):
    return torch.ones(shape, dtype=_dt(dtype) or torch.float32)


def zeros(shape, dtype=None):
    return torch.zeros(shape, dtype=_dt(dtype) or torch.float32)


def full(shape, value, dtype=None):
    return torch.full(shape, value, dtype=_dt(dtype) or torch.float32)


def arange(n, dtype=None):
    return torch.arange(n, dtype=_dt(dtype))


def tril(x):
    return torch.tril(x)


def concatenate(xs, axis=0):
    return torch.cat(list(xs), dim=axis)


def broadcast_to(x, shape):
    return torch.broadcast_to(_t(x), shape)


def take_along_axis(a, idx, axis=-1):
    n = a.shape[axis]
    idx = torch.where(idx < 0, idx + n, idx).long()
    return torch.gather(a, axis, idx)


def einsum(spec, a, b, preferred_element_type=None):
    d = torch.promote_types(a.dtype, b.dtype)
    if preferred_element_type is not None:
        d = torch.promote_types(d, _dt(preferred_element_type))
    return torch.einsum(spec, a.to(d), b.to(d))


def matmul(a, b, preferred_element_type=None):
    d = torch.promote_types(a.dtype, b.dtype)
    if preferred_element_type is not None:
        d = torch.promote_types(d, _dt(preferred_element_type))
    return a.to(d) @ b.to(d)


def arcsinh(x):
    return torch.asinh(x)


def log(x):
    return torch.log(x)


def exp(x):
    return torch.exp(x)


def sqrt(x):
    if not isinstance(x, torch.Tensor):  # a Python scalar: float64, the x64 setting of the goldens
        x = torch.tensor(float(x), dtype=torch.float64)
    return torch.sqrt(x)


def cos(x):
    return torch.cos(x)


def sin(x):
    return torch.sin(x)


def linspace(a, b, n, dtype=None):
    return torch.linspace(a, b, n, dtype=_dt(dtype) or torch.float32)


pi = 3.141592653589793


def square(x):
    return x * x


def swapaxes(x, a, b):
    return torch.swapaxes(x, a, b)


def eye(n, dtype=None):
    return torch.eye(n, dtype=_dt(dtype) or torch.float32)


def zeros_like(x):
    return torch.zeros_like(x)


def clip(x, lo, hi):
    return torch.clamp(x, min=lo, max=hi)
