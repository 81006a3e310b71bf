"""The config-5 language model: a pre-norm causal Transformer on the algx kernels.

Mirrors the reference's ``LMConfig`` / ``init_params`` / ``forward_hidden`` /
``head_loss`` (model.py:25-226) for the configuration its training-step
benchmark names: learned RMS gains, SwiGLU, RoPE, QK norm, causal
asinh-power attention with the range guard and a tied-embedding ``ce`` head;
and the reference's pure algebraic preset (ALU-GLU, geometric Cayley
rotations, a learned per-head sink, the ``alg_ce`` head). Per block (model.py:184-200):

    h  = rms_norm(x, ln1)
    qkv = h @ [w_q | w_k | w_v]                   one GEMM, token-major (B, T, 3, H, D)
    a  = attention(rot(qk_norm(q)), rot(qk_norm(k)), v)   read from qkv in place by the fused
                                                  prologue; tcgen05 kernels; output (B, T, H, D)
    x  = x + a @ w_o
    x  = x + glu(rms_norm(x, ln2) @ [w_g | w_u]) @ w_d      glu: SwiGLU or ALU-GLU

and each residual add runs fused into the RMS norm that reads its sum
(``add_rms_norm``: ln2 inside the block, the next block's ln1 or the final
gain after it).

Parameters are float32 masters; every matmul reads a bfloat16 copy of its
weight (``.astype(dt)`` in model.py:167-196), made once per weight version
rather than once per micro-batch, and its weight gradient comes out of the
GEMM in float32 and accumulates into the master's gradient. All parameters
live in two flat float32 buffers (decayed weights and
the embedding; gains and sinks), with every ``nn.Parameter`` a view into
them and every ``.grad`` a view into matching flat gradient buffers. The
optimizer then updates two tensors, the gradient all-reduce runs over
contiguous slices, and the global norm is two reductions.

Parameter names follow the reference's pytree (model.py:84-117), except that
``w_q, w_k, w_v`` are stored side by side as ``w_qkv`` (d, 3d) and
``w_g, w_u`` as ``w_gu`` (d, 2f): the concatenations the one-GEMM projections
read, with the same values and gradients column block by column block.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, replace
from typing import Dict, List, Optional, Tuple

import torch
from torch import nn

from . import rotary as R
from .kernels.flash import qknorm_flash_attention_packed
from .kernels.fused_head import fused_head
from .layers import add_rms_norm, aluglu, linear, rms_norm, swiglu

BF16 = torch.bfloat16


@dataclass(frozen=True)
class LMConfig:
    """The fields of model.py:25-61 that the algx model honours."""

    vocab_size: int = 50304
    d_model: int = 768
    n_layers: int = 12
    n_heads: int = 12
    d_ff: int = 2048
    seq_len: int = 2048
    eps: float = 1e-5
    ffn: str = "swiglu"          # "swiglu" or "alu_glu"
    alu_beta: float = 1.0
    pos: str = "rope"            # "rope" or "cayley_geo"
    rope_base: float = 10000.0
    rope_fraction: float = 1.0
    attn_n: int = 16
    attn_c: float = 8.0
    sink: str = "none"           # "none", "const" or "learned"
    sink_init: float = 0.0
    head: str = "ce"             # "ce" or "alg_ce"
    head_n: int = 16
    head_c: float = 16.0
    init_std: float = 0.02
    out_init_scale: float = 1.0

    @property
    def head_dim(self) -> int:
        return self.d_model // self.n_heads

    def validate(self) -> None:
        if self.d_model % self.n_heads:
            raise ValueError("d_model must be divisible by n_heads")
        if self.head_dim != 64:
            raise ValueError("the algx attention kernels need head_dim = 64")
        if self.ffn not in ("swiglu", "alu_glu"):
            raise ValueError(f"unknown ffn {self.ffn!r}")
        if self.pos not in ("rope", "cayley_geo"):
            raise ValueError(f"unknown position kind {self.pos!r}")
        if self.sink not in ("none", "const", "learned"):
            raise ValueError(f"unknown sink {self.sink!r}")
        if self.head not in ("ce", "alg_ce"):
            raise ValueError(f"unknown head {self.head!r}")


def config_125m(**overrides) -> LMConfig:
    """The training-step configuration: 125M size (config.py:10) with QK norm,
    asinh-power attention n=16, c=8 (config.py:33), RoPE, SwiGLU, the ``ce``
    head and a 50304-token vocabulary."""
    return replace(LMConfig(), **overrides)


_FIELD_TYPES = {"int": int, "float": float, "str": str, "bool": bool}


def parse_overrides(pairs) -> dict:
    """``key=value`` strings to typed ``LMConfig`` field overrides (the
    trainer's ``--set``, train.py:31-45): the value is converted by the
    field's declared type; booleans accept 1/true/yes (any case) as true.
    An unknown field raises ``ValueError``."""
    from dataclasses import fields
    types = {f.name: (f.type if isinstance(f.type, str) else f.type.__name__) for f in fields(LMConfig)}
    out = {}
    for item in pairs or []:
        key, _, value = item.partition("=")
        if key not in types:
            raise ValueError(f"unknown config field {key!r}")
        kind = _FIELD_TYPES[types[key]]
        out[key] = value.lower() in ("1", "true", "yes") if kind is bool else kind(value)
    return out


def config_algebraic_125m(**overrides) -> LMConfig:
    """The reference's pure algebraic preset at the 125M size (config.py:25-36):
    ALU-GLU with beta 1/2, geometric Cayley rotations, QK norm, rho(s/8)^16
    attention with a learned per-head sink, and the rho(z/2)^8 likelihood head."""
    return replace(LMConfig(ffn="alu_glu", alu_beta=0.5, pos="cayley_geo", sink="learned", sink_init=0.0,
                            head="alg_ce", head_n=8, head_c=2.0), **overrides)


@dataclass(frozen=True)
class ParamSpec:
    name: str
    shape: Tuple[int, ...]
    decay: bool      # weight matrices and the embedding (model.py:120-125)
    std: float       # 0 -> filled with `fill`
    fill: float = 0.0


def param_specs(cfg: LMConfig) -> List[ParamSpec]:
    """Every parameter, in the order the backward pass finishes them
    (final gain, last layer ... first layer, embedding gain, embedding), so
    that flat-buffer slices complete front to back during the backward."""
    d, f, H, D = cfg.d_model, cfg.d_ff, cfg.n_heads, cfg.head_dim
    s, so = cfg.init_std, cfg.init_std * cfg.out_init_scale
    specs = [ParamSpec("final_gain", (d,), False, 0.0, 1.0)]
    for i in reversed(range(cfg.n_layers)):
        p = f"layers.{i}."
        specs += [
            ParamSpec(p + "w_d", (f, d), True, so),
            ParamSpec(p + "w_gu", (d, 2 * f), True, s),
            ParamSpec(p + "ln2", (d,), False, 0.0, 1.0),
            ParamSpec(p + "w_o", (d, d), True, so),
            ParamSpec(p + "q_gain", (D,), False, 0.0, 1.0),
            ParamSpec(p + "k_gain", (D,), False, 0.0, 1.0),
        ]
        if cfg.sink == "learned":
            specs.append(ParamSpec(p + "sink", (H,), False, 0.0, cfg.sink_init))
        specs += [
            ParamSpec(p + "w_qkv", (d, 3 * d), True, s),
            ParamSpec(p + "ln1", (d,), False, 0.0, 1.0),
        ]
    specs += [ParamSpec("embed_gain", (d,), False, 0.0, 1.0),
              ParamSpec("embed", (cfg.vocab_size, d), True, s)]
    return specs


def count_params(cfg: LMConfig) -> int:
    return sum(math.prod(p.shape) for p in param_specs(cfg))


def train_flops_per_token(cfg: LMConfig) -> float:
    """6 P + 6 L S d: the matmul FLOPs of forward and backward per token
    (attention counted causally as half of 12 L S d)."""
    return 6.0 * count_params(cfg) + 6.0 * cfg.n_layers * cfg.seq_len * cfg.d_model


class FlatParams:
    """Two flat float32 buffers (decayed / not decayed) and their gradients.

    ``params[name]`` is an ``nn.Parameter`` whose storage is a slice of
    ``data[decay]`` and whose ``.grad`` is the same slice of ``grad[decay]``;
    autograd accumulates into those views in place. ``slices[name]`` gives
    (decay, start, end).
    """

    def __init__(self, specs: List[ParamSpec], device, generator: Optional[torch.Generator] = None):
        self.specs = specs
        sizes = {True: 0, False: 0}
        self.slices: Dict[str, Tuple[bool, int, int]] = {}
        for sp in specs:
            n = math.prod(sp.shape)
            self.slices[sp.name] = (sp.decay, sizes[sp.decay], sizes[sp.decay] + n)
            sizes[sp.decay] += n
        self.data = {k: torch.zeros(max(n, 1), dtype=torch.float32, device=device) for k, n in sizes.items()}
        self.grad = {k: torch.zeros_like(v) for k, v in self.data.items()}
        self.params: Dict[str, nn.Parameter] = {}
        for sp in specs:
            decay, a, b = self.slices[sp.name]
            view = self.data[decay][a:b].view(sp.shape)
            if sp.std > 0:
                noise = torch.randn(sp.shape, generator=generator, dtype=torch.float32)
                view.copy_(noise * sp.std)
            else:
                view.fill_(sp.fill)
            p = nn.Parameter(view)
            p.grad = self.grad[decay][a:b].view(sp.shape)
            self.params[sp.name] = p
        # the optimizer's view of the same storage: one tensor per group
        self.flat = {k: nn.Parameter(v) for k, v in self.data.items()}
        for k, v in self.flat.items():
            v.grad = self.grad[k]
        # optional callable(name), run before a parameter is handed out: a
        # sharded optimizer uses it to wait for the gather of that parameter's
        # updated values on first use
        self.fence = None

    def zero_grad(self) -> None:
        for g in self.grad.values():
            g.zero_()

    def __getitem__(self, name: str) -> nn.Parameter:
        if self.fence is not None:
            self.fence(name)
        return self.params[name]


class AlgebraicLM(nn.Module):
    """Config-5 model on the algx kernels (CUDA only, no fallback)."""

    def __init__(self, cfg: LMConfig, device="cuda", seed: int = 0):
        super().__init__()
        cfg.validate()
        self.cfg = cfg
        gen = torch.Generator().manual_seed(seed)
        self.flat = FlatParams(param_specs(cfg), device, gen)
        for name, p in self.flat.params.items():
            self.register_parameter(name.replace(".", "_"), p)
        T = cfg.seq_len
        if cfg.pos == "rope":
            cos, sin = R.rope_table(cfg.head_dim, T, cfg.rope_base, device=device)
        else:
            cos, sin = R.cayley_table_geometric(cfg.head_dim, T, cfg.rope_base, fraction=cfg.rope_fraction)
        self.register_buffer("rot_cos", cos.to(device=device, dtype=torch.float32).contiguous(), persistent=False)
        self.register_buffer("rot_sin", sin.to(device=device, dtype=torch.float32).contiguous(), persistent=False)
        self._w16 = {}

    def p(self, name: str) -> nn.Parameter:
        return self.flat[name]

    def weights_changed(self) -> None:
        """Drop the bf16 weight copies (the trainer calls this after each
        optimizer step to release them early)."""
        self._w16 = {}

    def _mm(self, x: torch.Tensor, name: str) -> torch.Tensor:
        """x @ bf16(w) with the bf16 copy made once per weight version: every
        parameter view shares its version counter with the flat buffer, so an
        optimizer step (or any in-place update) makes the next call recast."""
        w = self.flat[name]
        hit = self._w16.get(name)
        if hit is None or hit[0] != w._version:
            hit = self._w16[name] = (w._version, w.detach().to(BF16))
        return linear(x, w, hit[1])

    def _block(self, i: int, x: torch.Tensor, h: torch.Tensor):
        """Block i on the residual stream x with h = rms_norm(x, ln1) given;
        returns (x', rms_norm(x', next gain)), each residual add fused into the
        norm that follows it."""
        cfg = self.cfg
        B, T, d = x.shape
        H, D = cfg.n_heads, cfg.head_dim
        p = lambda n: self.flat[f"layers.{i}.{n}"]  # noqa: E731
        qkv = self._mm(h, f"layers.{i}.w_qkv").view(B, T, 3, H, D)  # token-major [q | k | v], no copy
        if cfg.sink == "learned":
            sink = p("sink")
        elif cfg.sink == "const":
            sink = torch.full((H,), cfg.sink_init, dtype=torch.float32, device=x.device)
        else:
            sink = None
        a = qknorm_flash_attention_packed(qkv, p("q_gain"), p("k_gain"), sink, eps=cfg.eps, kind="asinh",
                                          n=cfg.attn_n, c=cfg.attn_c, range_guard=True,
                                          rotary=(self.rot_cos, self.rot_sin))
        x, h2 = add_rms_norm(x, self._mm(a.view(B, T, d), f"layers.{i}.w_o"), p("ln2"), cfg.eps)
        gu = self._mm(h2, f"layers.{i}.w_gu")
        act = swiglu(gu) if cfg.ffn == "swiglu" else aluglu(gu, cfg.alu_beta)
        nxt = self.flat[f"layers.{i + 1}.ln1"] if i + 1 < cfg.n_layers else self.flat["final_gain"]
        return add_rms_norm(x, self._mm(act, f"layers.{i}.w_d"), nxt, cfg.eps)

    def forward_hidden(self, tokens: torch.Tensor) -> torch.Tensor:
        """Final normalised hidden states (B, T, d) in bf16 (model.py:203-215)."""
        cfg = self.cfg
        x = nn.functional.embedding(tokens, self.flat["embed"]).to(BF16)
        x = rms_norm(x, self.flat["embed_gain"], cfg.eps)
        h = rms_norm(x, self.flat["layers.0.ln1"], cfg.eps)
        for i in range(cfg.n_layers):
            x, h = self._block(i, x, h)
        return h

    def loss(self, tokens: torch.Tensor, targets: torch.Tensor):
        """(objective, telemetry) of one micro-batch (model.py:218-226, fused head)."""
        cfg = self.cfg
        hidden = self.forward_hidden(tokens)
        N = hidden.shape[0] * hidden.shape[1]
        return fused_head(hidden.reshape(N, -1), self.flat["embed"], targets.reshape(N), kind=cfg.head,
                          n=cfg.head_n, c=cfg.head_c)
