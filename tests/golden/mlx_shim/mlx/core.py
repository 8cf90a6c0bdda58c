"""Test-only stand-in for ``mlx.core`` over torch-CPU.

MLX cannot be installed in this environment (no wheel, no network), so the
golden-vector generator imports the reference's own, unmodified Python
(``mlx_gsplat/rendering.py``, ``optimizer.py``, ``allocator.py``) with this
module registered as ``mlx.core``.  It covers exactly the operations those
files use, with MLX's conventions where they differ from torch's:

* ``mx.array`` of float64 data becomes float32 (MLX has no float64 compute);
  integer ``arange`` is int32.
* ``maximum``/``minimum``/``clip`` carry MLX's VJP tie rule: for
  ``maximum(a, b)`` the gradient goes to ``a`` where ``a > b`` and to ``b``
  elsewhere (``minimum``: ``a < b``).  ``clip`` is ``minimum(maximum(x, lo), hi)``.
* ``value_and_grad`` returns zeros (not ``None``) for inputs the loss does not
  touch, as MLX does.

This is the checker's scaffolding only; nothing in the product imports it.
"""
import builtins as _bi

import numpy as _np
import torch as _torch

float32 = _torch.float32
float16 = _torch.float16
int32 = _torch.int32
int64 = _torch.int64
uint32 = _torch.int64  # argsort results; only used as indices
bool_ = _torch.bool
globals()["bool"] = _torch.bool

_GEN = _torch.Generator().manual_seed(0)
_NORMAL_LOG = []  # every mx.random.normal draw, so a caller can replay it


def _t(x, dtype=None):
    if isinstance(x, _torch.Tensor):
        out = x
    else:
        out = _torch.as_tensor(_np.asarray(x))
    if dtype is not None:
        out = out.to(dtype)
    elif out.dtype == _torch.float64:
        out = out.to(_torch.float32)
    return out


def array(x, dtype=None):
    if isinstance(x, _torch.Tensor):
        return _t(x.detach().clone(), dtype)
    if isinstance(x, (float, int, _bi.bool)) and dtype is None:
        if isinstance(x, _bi.bool):
            return _torch.tensor(x)
        if isinstance(x, int):
            return _torch.tensor(x, dtype=_torch.int32)
        return _torch.tensor(x, dtype=_torch.float32)
    return _t(x, dtype).clone()


def zeros(shape, dtype=float32):
    return _torch.zeros(shape, dtype=dtype)


def ones(shape, dtype=float32):
    return _torch.ones(shape, dtype=dtype)


def full(shape, val, dtype=None):
    out = _torch.full(tuple(shape) if not isinstance(shape, int) else (shape,), float(val))
    return out if dtype is None else out.to(dtype)


def zeros_like(a):
    return _torch.zeros_like(a)


def ones_like(a):
    return _torch.ones_like(a)


def arange(*args, dtype=None):
    if dtype is None:
        dtype = int32 if all(isinstance(a, int) for a in args) else float32
    return _torch.arange(*args, dtype=dtype)


def take(a, idx, axis=None):
    idx = _t(idx).long()
    if axis is None:
        return a.reshape(-1)[idx]
    return _torch.index_select(a, axis, idx.reshape(-1)).reshape(
        a.shape[:axis] + idx.shape + a.shape[axis + 1:])


def matmul(a, b):
    return _torch.matmul(a, b)


def concatenate(xs, axis=0):
    return _torch.cat(list(xs), dim=axis)


def stack(xs, axis=0):
    return _torch.stack(list(xs), dim=axis)


def where(c, a, b):
    a = a if isinstance(a, _torch.Tensor) else _torch.tensor(a, dtype=float32)
    b = b if isinstance(b, _torch.Tensor) else _torch.tensor(b, dtype=float32)
    return _torch.where(c, a, b)


def sort(a, axis=-1):
    return _torch.sort(a, dim=axis, stable=True).values


def argsort(a, axis=-1):
    return _torch.argsort(a, dim=axis, stable=True)


def sum(a, axis=None, keepdims=False):  # noqa: A001 - MLX name
    if axis is None:
        return _torch.sum(a)
    return _torch.sum(a, dim=axis, keepdim=keepdims)


def mean(a, axis=None, keepdims=False):
    if axis is None:
        return _torch.mean(a)
    return _torch.mean(a, dim=axis, keepdim=keepdims)


def abs(a):  # noqa: A001
    return _torch.abs(a)


def sqrt(a):
    return _torch.sqrt(a)


def exp(a):
    return _torch.exp(a)


def sigmoid(a):
    return _torch.sigmoid(a)


def floor(a):
    return _torch.floor(a)


def transpose(a, axes=None):
    if axes is None:
        axes = tuple(reversed(range(a.dim())))
    return a.permute(*axes)


def expand_dims(a, axis):
    return _torch.unsqueeze(a, axis)


def cumprod(a, axis=None):
    return _torch.cumprod(a, dim=axis)


def meshgrid(*xs, indexing="xy"):
    return _torch.meshgrid(*xs, indexing=indexing)


class _MaxMLX(_torch.autograd.Function):
    @staticmethod
    def forward(ctx, a, b):
        ctx.save_for_backward(a, b)
        return _torch.where(a > b, a, b)

    @staticmethod
    def backward(ctx, g):
        a, b = ctx.saved_tensors
        m = (a > b).to(g.dtype)
        ga = g * m
        gb = g * (1 - m)
        return _red(ga, a.shape), _red(gb, b.shape)


class _MinMLX(_torch.autograd.Function):
    @staticmethod
    def forward(ctx, a, b):
        ctx.save_for_backward(a, b)
        return _torch.where(a < b, a, b)

    @staticmethod
    def backward(ctx, g):
        a, b = ctx.saved_tensors
        m = (a < b).to(g.dtype)
        return _red(g * m, a.shape), _red(g * (1 - m), b.shape)


def _red(g, shape):
    # sum a broadcast gradient back to an operand's shape
    while g.dim() > len(shape):
        g = g.sum(0)
    for i, s in enumerate(shape):
        if s == 1 and g.shape[i] != 1:
            g = g.sum(i, keepdim=True)
    return g


def _as_operand(x, like):
    if isinstance(x, _torch.Tensor):
        return x
    return _torch.tensor(x, dtype=like.dtype)


def maximum(a, b):
    if not isinstance(a, _torch.Tensor):
        a, b = b, a
    return _MaxMLX.apply(a, _as_operand(b, a))


def minimum(a, b):
    if not isinstance(a, _torch.Tensor):
        a, b = b, a
    return _MinMLX.apply(a, _as_operand(b, a))


def clip(a, a_min=None, a_max=None):
    out = a
    if a_min is not None:
        out = maximum(out, a_min)
    if a_max is not None:
        out = minimum(out, a_max)
    return out


def conv2d(x, w, stride=1, padding=0, groups=1):
    # MLX: x NHWC, w [C_out, kH, kW, C_in/groups]
    y = _torch.nn.functional.conv2d(x.permute(0, 3, 1, 2), w.permute(0, 3, 1, 2),
                                    stride=stride, padding=padding, groups=groups)
    return y.permute(0, 2, 3, 1)


def eval(*args):  # noqa: A001
    return None


def clear_cache():
    return None


def value_and_grad(fn):
    def wrapped(params):
        leaves = {k: v.detach().clone().requires_grad_(True) for k, v in params.items()}
        out = fn(leaves)
        names = list(leaves.keys())
        grads = _torch.autograd.grad(out, [leaves[k] for k in names], allow_unused=True)
        gd = {}
        for k, g in zip(names, grads):
            gd[k] = _torch.zeros_like(leaves[k]) if g is None else g.detach()
        return out.detach(), gd
    return wrapped


class _Random:
    @staticmethod
    def normal(shape, dtype=float32):
        out = _torch.randn(tuple(shape), generator=_GEN, dtype=dtype)
        _NORMAL_LOG.append(out.clone())
        return out

    @staticmethod
    def seed(s):
        _GEN.manual_seed(int(s))


random = _Random()


def _install_tensor_methods():
    """MLX array methods that torch tensors lack (``astype``) and numpy's
    ``copy=False`` conversion used by the reference's pointer caching."""
    if not hasattr(_torch.Tensor, "astype"):
        _torch.Tensor.astype = lambda self, dt: self.to(dt)
    orig = _torch.Tensor.__array__

    def _arr(self, dtype=None, copy=None):
        a = self.detach().numpy()
        if dtype is not None:
            a = a.astype(dtype)
        return a.copy() if copy else a
    if getattr(orig, "__name__", "") != "_arr":
        _torch.Tensor.__array__ = _arr


_install_tensor_methods()
