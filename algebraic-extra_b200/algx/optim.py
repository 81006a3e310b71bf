"""The reference trainer's optimizers on torch tensors (optimizers.py:1-248):
Muon on the 2-D weight matrices + AdamW on the rest (``muon_adamw``),
cautious AdamW everywhere (``cadamw``), and Muon + cautious AdamW
(``hybrid_muon_cadamw``), with the cosine learning-rate schedule.

The update rules are the reference's, element for element; the schedule and
the Adam bias corrections are computed in float32 as the reference computes
them. Parameters are addressed by name: the reference's routing rule
(``is_muon_param``, optimizers.py:68-89) reads the last path component, and a
weight the model stores fused (``w_qkv`` = [w_q | w_k | w_v], ``w_gu`` =
[w_g | w_u], column blocks) is updated block by block, so each reference
matrix gets its own Newton-Schulz orthogonalisation and its own cautious mask
mean.

Two interfaces share the same update rules: ``get_optimizer`` (init_fn,
step_fn over trees of tensors, the reference's own functional interface,
optimizers.py:118-240) and ``ReferenceOptimizer`` (in place over named
parameters with ``.grad``, stacked by shape, optionally sharded over ranks;
what the data-parallel trainer uses).
"""

from __future__ import annotations

import math
from typing import Any, Iterable, List, NamedTuple, Optional, Tuple

import torch
import torch.distributed as dist

# Quintic Newton-Schulz coefficients of the Muon optimizer (optimizers.py:38)
NS_COEFFS = (3.4445, -4.7750, 2.0315)
NAMES = ("muon_adamw", "cadamw", "hybrid_muon_cadamw")


PRECISIONS = ("highest", "default")


def _matmul_ops(precision: str, like: torch.Tensor):
    """(round an operand, multiply rounded operands) for a matmul precision.

    ``highest``: operands and products in the working dtype. ``default``:
    operands rounded to bf16, products accumulated in float32, which is what
    XLA's DEFAULT precision computes for a float32 dot on the TPU the
    reference trains on; on a CUDA float32 tensor it runs on the bf16 tensor
    cores with a float32 output."""
    if precision == "highest":
        return (lambda t: t), torch.matmul
    if precision != "default":
        raise ValueError(f"unknown matmul precision {precision!r}; choices: {PRECISIONS}")
    if like.is_cuda and like.dtype == torch.float32:
        def mm(a, b):
            f = torch.bmm if a.ndim == 3 else torch.mm
            return f(a, b, out_dtype=torch.float32)
        return (lambda t: t.to(torch.bfloat16)), mm
    dt = like.dtype
    return (lambda t: t.to(torch.bfloat16).to(dt)), torch.matmul


def _ns_iterations_tensor_cores(X: torch.Tensor, steps: int) -> torch.Tensor:
    """The iterations of newton_schulz_5 at ``default`` precision on a CUDA
    float32 batch (count, m, n), m <= n: bf16 operands on the tensor cores,
    float32 products, with each linear combination folded into the product
    that feeds it (beta * C + alpha * A @ B in the GEMM epilogue):
    B = b A + c A^2, X <- a X + B X, and the refinement as
    X <- 1.5 X - 0.5 A X. The operands are rounded to bf16 as in the literal
    sequence; the result differs from it only at that rounding level, and it
    saves the separate element-wise passes over the stacks."""
    a, b, c = NS_COEFFS
    f32, bf16 = torch.float32, torch.bfloat16
    fma_mm = torch.ops.aten.baddbmm.dtype
    for _ in range(steps):
        x = X.to(bf16)
        A = torch.bmm(x, x.transpose(-2, -1), out_dtype=f32)
        a16 = A.to(bf16)
        B = fma_mm(A, a16, a16, f32, beta=b, alpha=c)
        X = fma_mm(X, B.to(bf16), x, f32, beta=a, alpha=1.0)
    for _ in range(2):
        x = X.to(bf16)
        A = torch.bmm(x, x.transpose(-2, -1), out_dtype=f32)
        X = fma_mm(X, A.to(bf16), x, f32, beta=1.5, alpha=-0.5)
    return X


def newton_schulz_5(G: torch.Tensor, steps: int = 5, eps: float = 1e-7, precision: str = "highest") -> torch.Tensor:
    """Orthogonalise the trailing two dimensions of G (optimizers.py:27-65):
    Frobenius pre-normalisation, ``steps`` quintic iterations, two order-3
    Schulz refinements, then scaling by sqrt(max(1, M / N)). The Gram
    matrices are min(M, N) square (G is transposed first when M > N).
    Leading dimensions are a batch of independent matrices."""
    if G.ndim < 2:
        return G
    if G.ndim > 3:
        return newton_schulz_5(G.reshape(-1, *G.shape[-2:]), steps, eps, precision).reshape(G.shape)
    lo, mm = _matmul_ops(precision, G)
    a, b, c = NS_COEFFS
    M, N = G.shape[-2], G.shape[-1]
    transposed = M > N
    X = G.transpose(-2, -1) if transposed else G
    X = X / torch.sqrt(torch.sum(X * X, dim=(-2, -1), keepdim=True) + eps)
    if precision == "default" and X.is_cuda and X.dtype == torch.float32:
        X = _ns_iterations_tensor_cores(X if X.ndim == 3 else X.unsqueeze(0), steps).reshape(X.shape)
        if transposed:
            X = X.transpose(-2, -1)
        return X * math.sqrt(max(1.0, float(M) / float(N)))
    for _ in range(steps):
        x = lo(X)
        A = mm(x, x.transpose(-2, -1))
        a16 = lo(A)
        B = b * A + c * mm(a16, a16)
        X = a * X + mm(lo(B), x)
    eye = torch.eye(min(M, N), dtype=X.dtype, device=X.device)
    for _ in range(2):
        x = lo(X)
        A = mm(x, x.transpose(-2, -1))
        X = 0.5 * mm(lo(3.0 * eye - A), x)
    if transposed:
        X = X.transpose(-2, -1)
    return X * math.sqrt(max(1.0, float(M) / float(N)))


def is_muon_param(path, param) -> bool:
    """The reference's routing (optimizers.py:68-89) on the last path
    component: ``path`` is a dotted name or a sequence of keys (a key object
    with a ``key`` attribute counts by that attribute, as in the reference),
    ``param`` a tensor or its number of dimensions."""
    ndim = param if isinstance(param, int) else getattr(param, "ndim", 0)
    if isinstance(path, str):
        key = path.split(".")[-1]
    elif path:
        last = path[-1]
        key = str(getattr(last, "key", last))
    else:
        key = ""
    if key == "embed":
        return False
    if key.startswith("w_"):
        return True
    if key.startswith("ln") or key.endswith("_gain") or key == "sink" or "bias" in key:
        return False
    return ndim >= 2


def cosine_schedule(peak_lr: float, total_steps: int, warmup_fraction: float, min_lr_ratio: float):
    """Linear warm-up then cosine decay to peak * min_lr_ratio (optimizers.py:92-115),
    in float32 like the reference."""
    f32 = torch.float32
    warm = float(warmup_fraction) if warmup_fraction >= 1 else max(1.0, float(round(warmup_fraction * total_steps)))
    floor = peak_lr * min_lr_ratio

    def lr(step: int) -> torch.Tensor:
        t = torch.tensor(float(step), dtype=f32) + 1.0
        warm_f = torch.clamp(t / warm, max=1.0)
        prog = torch.clamp((t - warm) / max(1.0, float(total_steps) - warm), 0.0, 1.0)
        cos = floor + (peak_lr - floor) * 0.5 * (1.0 + torch.cos(math.pi * prog))
        return torch.where(t < warm, peak_lr * warm_f, cos)

    return lr


def reference_blocks(name: str, param: torch.Tensor) -> List[Tuple[str, torch.Tensor]]:
    """The reference parameters a (possibly fused) model parameter holds, as views."""
    key = name.split(".")[-1]
    base = name[: len(name) - len(key)]
    if key == "w_qkv":
        d = param.shape[1] // 3
        return [(base + k, param[:, i * d:(i + 1) * d]) for i, k in enumerate(("w_q", "w_k", "w_v"))]
    if key == "w_gu":
        f = param.shape[1] // 2
        return [(base + k, param[:, i * f:(i + 1) * f]) for i, k in enumerate(("w_g", "w_u"))]
    return [(name, param)]


make_cosine_schedule = cosine_schedule  # the reference's name (optimizers.py:92)


def _step_scalars(step: int, adam_lr, muon_lr, b1: float, b2: float, wd: float, muon_wd: float):
    """The step's float32 host quantities as exact Python floats: bias
    corrections 1 - b^t (t = step + 1), the two learning rates and the two
    decay factors 1 - lr * wd (optimizers.py:179-184, 215, 225, 233)."""
    f32 = torch.float32
    t = torch.tensor(float(step + 1), dtype=f32)
    c1 = float(1.0 - torch.tensor(b1, dtype=f32) ** t)
    c2 = float(1.0 - torch.tensor(b2, dtype=f32) ** t)
    lr_a_t, lr_m_t = adam_lr(step), muon_lr(step)
    return (c1, c2, float(lr_a_t), float(lr_m_t), float(1.0 - lr_a_t * wd), float(1.0 - lr_m_t * muon_wd))


def _muon_update(p, g, m, mu: float, decay: float, lr: float, ns_steps: int, precision: str, matrix: bool):
    """Muon on a stack of parameters (optimizers.py:210-219): momentum m
    updated in place, Newton-Schulz of the Nesterov combination (a vector
    passes through), returns the new parameters."""
    m.mul_(mu).add_((1.0 - mu) * g)
    x = (1.0 - mu) * g + mu * m
    o = newton_schulz_5(x, steps=ns_steps, precision=precision) if matrix else x
    return p * decay - lr * o


def _adam_update(p, g, m, v, b1: float, b2: float, c1: float, c2: float, eps: float, cautious_eps: Optional[float],
                 decay: float, lr: float):
    """AdamW, or cautious AdamW when ``cautious_eps`` is given, on a stack of
    parameters (optimizers.py:220-238): m and v updated in place, the
    cautious mask's mean taken per row of the stack; returns the new
    parameters."""
    m.mul_(b1).add_((1.0 - b1) * g)
    v.mul_(b2).add_((1.0 - b2) * (g * g))
    u = (m / c1) / (torch.sqrt(v / c2) + eps)
    if cautious_eps is not None:  # keep the components that agree with the gradient
        # the reference's 0/1 mask is built from Python scalars: float32
        mask = (u * g > 0.0).to(torch.float32)
        mean = mask.mean(dim=tuple(range(1, mask.ndim)), keepdim=True) if mask.ndim > 1 else mask
        u = u * (mask / torch.clamp(mean, min=cautious_eps))
    return p * decay - lr * u


class _Group:
    """Reference parameters of one shape, dtype and routing, updated together:
    their values and gradients are gathered into one (count, *shape) stack
    per step, the optimizer state lives stacked, and every per-matrix
    quantity (the Newton-Schulz normalisation, the cautious mask's mean) is
    taken per row of the stack."""

    def __init__(self, shape, decayed: bool, muon: bool, like: torch.Tensor):
        self.shape, self.decayed, self.muon = tuple(shape), decayed, muon
        self.like = like
        self.params: List[torch.Tensor] = []
        self.grads: List[torch.Tensor] = []
        self.names: List[str] = []
        self.m = self.v = None

    def add(self, name: str, p: torch.Tensor, g: torch.Tensor) -> None:
        self.names.append(name)
        self.params.append(p)
        self.grads.append(g)

    def init_state(self, rank: int = 0, world: int = 1) -> None:
        """State for the rows this rank updates: all of them (world 1), or a
        contiguous share of ceil(n / world) rows, padded with zero rows so that
        every rank's share has the same size for the all-gather."""
        n = len(self.params)
        self.world = world
        self.chunk = n if world == 1 else -(-n // world)
        self.lo = min(n, rank * self.chunk) if world > 1 else 0
        self.hi = min(n, self.lo + self.chunk)
        self.m = torch.zeros((self.chunk,) + self.shape, dtype=self.like.dtype, device=self.like.device)
        self.v = None if self.muon else torch.zeros_like(self.m)

    def own_stack(self, tensors: List[torch.Tensor]) -> torch.Tensor:
        """This rank's rows of ``tensors`` stacked, zero rows after them up to
        the share size (zero rows update to zero: no division by zero)."""
        own = tensors[self.lo:self.hi]
        if len(own) == self.chunk:
            return torch.stack(own)
        out = torch.zeros((self.chunk,) + self.shape, dtype=self.like.dtype, device=self.like.device)
        if own:
            out[:len(own)] = torch.stack(own)
        return out


class ReferenceOptimizer:
    """One of the reference's optimizers over named parameters (with .grad).

    ``params``: (name, tensor, decayed) triples; the tensors are updated in
    place. ``step(step)`` applies the update for the 0-based step index, with
    the learning rates of the reference's schedules (optimizers.py:153-154).
    ``precision`` is the Newton-Schulz matmul precision (``highest`` or
    ``default``, see ``_matmul_ops``). ``shard``: the ranks of ``group`` (a
    torch.distributed process group whose ranks hold the same parameters and
    gradients) split every Muon stack of at least as many matrices as ranks,
    each orthogonalising a contiguous share, and all-gather the updated
    matrices; the other stacks are updated on every rank.
    """

    def __init__(self, name: str, params: Iterable[Tuple[str, torch.Tensor, bool]], lr: float,
                 weight_decay: float = 0.1, total_steps: int = 1000, warmup_fraction: float = 0.02,
                 min_lr_ratio: float = 0.1, b1: float = 0.9, b2: float = 0.95, adam_eps: float = 1e-8,
                 muon_lr: Optional[float] = None, muon_wd: Optional[float] = None, muon_momentum: float = 0.95,
                 muon_steps: int = 5, cautious_eps: float = 1e-3, precision: str = "highest",
                 shard: bool = False, group=None):
        name = name.lower().strip()
        if name not in NAMES:
            raise ValueError(f"Unknown optimizer: {name}. Choices: {NAMES}")
        if precision not in PRECISIONS:
            raise ValueError(f"unknown matmul precision {precision!r}; choices: {PRECISIONS}")
        self.name = name
        self.precision = precision
        self.wd = weight_decay
        self.muon_wd = weight_decay if muon_wd is None else muon_wd
        self.b1, self.b2, self.eps = b1, b2, adam_eps
        self.mu, self.ns_steps, self.cautious_eps = muon_momentum, muon_steps, cautious_eps
        self.adam_lr = cosine_schedule(lr, total_steps, warmup_fraction, min_lr_ratio)
        self.muon_lr = cosine_schedule(lr if muon_lr is None else muon_lr, total_steps, warmup_fraction,
                                       min_lr_ratio)
        groups = {}
        for pname, p, decayed in params:
            if p.grad is None:
                raise ValueError(f"parameter {pname} has no .grad buffer")
            for (bname, pv), (_, gv) in zip(reference_blocks(pname, p.data), reference_blocks(pname, p.grad)):
                muon = name != "cadamw" and is_muon_param(bname, pv.ndim)
                key = (tuple(pv.shape), bool(decayed), muon, pv.dtype, pv.device)
                if key not in groups:
                    groups[key] = _Group(pv.shape, bool(decayed), muon, pv)
                groups[key].add(bname, pv, gv)
        self.groups: List[_Group] = list(groups.values())
        self.pg = group
        world = dist.get_world_size(group) if shard and dist.is_available() and dist.is_initialized() else 1
        rank = dist.get_rank(group) if world > 1 else 0
        self.sharded_groups = 0
        for grp in self.groups:
            split = grp.muon and world > 1 and len(grp.params) >= world
            grp.init_state(rank, world if split else 1)
            self.sharded_groups += int(split)

    @torch.no_grad()
    def step(self, step: int) -> None:
        # The schedule, bias corrections and decay factors are float32
        # arithmetic, as in the reference, done on the host; their exact
        # float32 values reach the device ops as Python scalars. (A 0-d host
        # tensor moved to the device would be a pageable copy, which can hold
        # the host until the stream drains and then expose every launch of the
        # update.)
        c1, c2, lr_a, lr_m, decay_a, decay_m = _step_scalars(step, self.adam_lr, self.muon_lr, self.b1, self.b2,
                                                             self.wd, self.muon_wd)
        cautious = self.cautious_eps if self.name != "muon_adamw" else None
        for grp in self.groups:
            dev = grp.m.device
            g = grp.own_stack(grp.grads)
            p = grp.own_stack(grp.params)
            if grp.muon:
                p = _muon_update(p, g, grp.m, self.mu, decay_m if grp.decayed else 1.0, lr_m, self.ns_steps,
                                 self.precision, len(grp.shape) >= 2)
            else:
                p = _adam_update(p, g, grp.m, grp.v, self.b1, self.b2, c1, c2, self.eps, cautious,
                                 decay_a if grp.decayed else 1.0, lr_a)
            if grp.world > 1:
                full = torch.empty((grp.world * grp.chunk,) + grp.shape, dtype=p.dtype, device=dev)
                dist.all_gather_into_tensor(full, p.contiguous(), group=self.pg)
                p = full[:len(grp.params)]
            torch._foreach_copy_(grp.params, list(p.unbind(0)))


# ------------------------------------------------- the reference's interface
class OptState(NamedTuple):
    """Optimizer state of ``get_optimizer`` (optimizers.py:19-24): the step
    count, and first / second moments as trees shaped like the parameters
    (second moment None for the parameters Muon updates)."""
    count: torch.Tensor
    m: Any
    v: Any


def _tree_map(fn, n_out: int, path: tuple, *trees):
    """Apply fn(path, *leaves) -> n_out-tuple over matching nested dicts /
    lists / tuples; returns n_out trees of the same structure."""
    t0 = trees[0]
    if isinstance(t0, dict):
        sub = {k: _tree_map(fn, n_out, path + (k,), *(t[k] for t in trees)) for k in t0}
        return tuple({k: sub[k][i] for k in t0} for i in range(n_out))
    if isinstance(t0, (list, tuple)):
        sub = [_tree_map(fn, n_out, path + (j,), *(t[j] for t in trees)) for j in range(len(t0))]
        return tuple(type(t0)(x[i] for x in sub) for i in range(n_out))
    return fn(path, *trees)


def _leaf_name(path: tuple) -> str:
    return ".".join(str(k) for k in path)


def get_optimizer(name: str, lr: float, weight_decay: float = 0.1, total_steps: int = 1000,
                  warmup_fraction: float = 0.02, min_lr_ratio: float = 0.1, b1: float = 0.9, b2: float = 0.95,
                  adam_eps: float = 1e-8, muon_lr: Optional[float] = None, muon_wd: Optional[float] = None,
                  muon_momentum: float = 0.95, muon_steps: int = 5, cautious_eps: float = 1e-3,
                  precision: str = "highest", **kwargs: Any):
    """(init_fn, step_fn) with the reference's signatures and names
    (optimizers.py:118-240), over trees (nested dicts, lists, tuples) of
    torch tensors: ``init_fn(params) -> OptState``;
    ``step_fn(step, params, grads, opt_state, decay_mask) -> (params, OptState)``,
    functional (its inputs are not modified). Routing by the last path
    component; a leaf named ``w_qkv`` or ``w_gu`` is updated as its reference
    matrices. ``precision``: the Newton-Schulz matmul precision. Unknown
    names raise ``ValueError`` with the reference's message."""
    opt_name = name.lower().strip()
    if opt_name not in NAMES:
        raise ValueError(f"Unknown optimizer: {name}. Choices: {NAMES}")
    if precision not in PRECISIONS:
        raise ValueError(f"unknown matmul precision {precision!r}; choices: {PRECISIONS}")
    actual_muon_wd = weight_decay if muon_wd is None else muon_wd
    adam_schedule = cosine_schedule(lr, total_steps, warmup_fraction, min_lr_ratio)
    muon_schedule = cosine_schedule(lr if muon_lr is None else muon_lr, total_steps, warmup_fraction, min_lr_ratio)
    cautious = cautious_eps if opt_name != "muon_adamw" else None

    def uses_muon(bname: str, p: torch.Tensor) -> bool:
        return opt_name != "cadamw" and is_muon_param(bname, p.ndim)

    def init_fn(params) -> OptState:
        def leaf(path, p):
            v = torch.zeros_like(p)
            blocks = reference_blocks(_leaf_name(path), p)
            return torch.zeros_like(p), (None if all(uses_muon(b, pv) for b, pv in blocks) else v)
        m, v = _tree_map(leaf, 2, (), params)
        return OptState(count=torch.zeros((), dtype=torch.int32), m=m, v=v)

    def step_fn(step, params, grads, opt_state: OptState, decay_mask):
        step = int(step)
        c1, c2, lr_a, lr_m, decay_a, decay_m = _step_scalars(step, adam_schedule, muon_schedule, b1, b2,
                                                             weight_decay, actual_muon_wd)

        def leaf(path, p, g, m, v, d):
            p_new, m_new = p.clone(), m.clone()
            v_new = None if v is None else v.clone()
            d = bool(d)
            name_ = _leaf_name(path)
            for (bname, pb), (_, gb), (_, mb) in zip(reference_blocks(name_, p_new), reference_blocks(name_, g),
                                                     reference_blocks(name_, m_new)):
                # each reference matrix as a stack of one
                if uses_muon(bname, pb):
                    upd = _muon_update(pb.unsqueeze(0), gb.unsqueeze(0), mb.unsqueeze(0), muon_momentum,
                                       decay_m if d else 1.0, lr_m, muon_steps, precision, pb.ndim >= 2)
                else:
                    vb = dict(reference_blocks(name_, v_new))[bname]
                    upd = _adam_update(pb.unsqueeze(0), gb.unsqueeze(0), mb.unsqueeze(0), vb.unsqueeze(0), b1, b2,
                                       c1, c2, adam_eps, cautious, decay_a if d else 1.0, lr_a)
                pb.copy_(upd[0])
            return p_new, m_new, v_new

        with torch.no_grad():
            p, m, v = _tree_map(leaf, 3, (), params, grads, opt_state.m, opt_state.v, decay_mask)
        return p, OptState(count=opt_state.count + 1, m=m, v=v)

    return init_fn, step_fn
