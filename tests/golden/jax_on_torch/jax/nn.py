"""``jax.nn`` subset on torch (fixture generation only)."""

import torch


def sigmoid(x):
    return torch.sigmoid(x)


def logsumexp(x, axis=-1):
    return torch.logsumexp(x, dim=axis)


def softmax(x, axis=-1):
    return torch.softmax(x, dim=axis)


def log_softmax(x, axis=-1):
    return torch.log_softmax(x, dim=axis)
