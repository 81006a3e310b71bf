"""A torch-CPU stand-in for the slice of JAX that the reference's dense maths uses.

Fixture generation only (``tests/golden/make_golden.py``): it lets this
container execute the reference's own ``algebraic.py``, ``standard.py``,
``evaluation.py`` and ``optimizers.py`` source without JAX, which is not installed here. Arrays are
torch tensors; ``jax.custom_vjp`` becomes a ``torch.autograd.Function`` that
calls the reference's own forward/backward rules, and plain autodiff becomes
torch autograd. Nothing outside ``tests/golden/make_golden.py`` imports it.
"""

import torch

from . import lax, nn, numpy, tree_util  # noqa: F401

Array = torch.Tensor


class _Config:
    def update(self, *_args, **_kwargs):
        return None


config = _Config()


class custom_vjp:
    """``jax.custom_vjp`` on top of ``torch.autograd.Function``."""

    def __init__(self, fun, nondiff_argnums=()):
        self.fun = fun
        self.nondiff = tuple(nondiff_argnums)
        self.fwd = None
        self.bwd = None

    def defvjp(self, fwd, bwd):
        self.fwd, self.bwd = fwd, bwd

    def __call__(self, *args):
        if self.fwd is None or not torch.is_grad_enabled():
            return self.fun(*args)
        owner = self
        diff = [i for i in range(len(args)) if i not in self.nondiff]

        class _Fn(torch.autograd.Function):
            @staticmethod
            def forward(ctx, *flat):
                full = list(args)
                for i, t in zip(diff, flat):
                    full[i] = t
                out, res = owner.fwd(*full)
                ctx.res = res
                ctx.is_tuple = isinstance(out, tuple)
                return tuple(out) if ctx.is_tuple else out

            @staticmethod
            def backward(ctx, *gouts):
                g = tuple(gouts) if ctx.is_tuple else gouts[0]
                nd = [args[i] for i in owner.nondiff]
                cot = owner.bwd(*nd, ctx.res, g)
                return tuple(cot)

        return _Fn.apply(*[args[i] for i in diff])
