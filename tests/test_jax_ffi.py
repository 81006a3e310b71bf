"""The JAX front-end (algx_jax + jax_ffi/algx_jax_ffi.cc).

jaxlib is not installed in this image, so the checks that need it skip; the
rest hold without it: every FFI target the shims register has a handler, the
handlers call only entry points the C ABI declares, the shims keep the
reference's signatures (the torch front-end's, which mirror the reference)
and resolve variants through the same torch-free module.
"""

import ast
import importlib.util
import inspect
import os
import re
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "algebraic-extra_b200")
CC = os.path.join(PKG, "jax_ffi", "algx_jax_ffi.cc")
SHIMS = os.path.join(PKG, "algx_jax")
HAS_JAX = importlib.util.find_spec("jax") is not None


def _declared():
    text = open(os.path.join(ROOT, "include", "algx.h")).read()
    return set(re.findall(r"ALGX_API\s+[\w\s\*]+?\b(algx_\w+)\s*\(", text))


def _targets():
    tree = ast.parse(open(os.path.join(SHIMS, "_ffi.py")).read())
    for node in ast.walk(tree):
        if isinstance(node, ast.Assign) and any(getattr(t, "id", "") == "TARGETS" for t in node.targets):
            return ast.literal_eval(node.value)
    raise AssertionError("TARGETS not found")


def test_every_registered_target_has_a_handler():
    text = open(CC).read()
    handlers = set(re.findall(r"XLA_FFI_DEFINE_HANDLER_SYMBOL\((\w+),", text))
    targets = _targets()
    assert set(targets.values()) == handlers
    called = set()
    for f in os.listdir(SHIMS):
        if f.endswith(".py"):
            called |= set(re.findall(r'ffi_call\(\s*"(\w+)"', open(os.path.join(SHIMS, f)).read()))
    assert called == set(targets), (called, set(targets))


def test_handlers_call_only_declared_entry_points():
    text = open(CC).read()
    used = set(re.findall(r"\b(algx_\w+)\s*\(", text))
    assert used <= _declared(), used - _declared()
    assert {"algx_attn_prepare", "algx_attn_fwd", "algx_attn_bwd", "algx_head_fwd", "algx_head_bwd",
            "algx_qknorm_fwd", "algx_qknorm_bwd"} <= used


def _shim_signature(module, name):
    tree = ast.parse(open(os.path.join(SHIMS, module + ".py")).read())
    for node in tree.body:
        if isinstance(node, ast.FunctionDef) and node.name == name:
            a = node.args
            pos = [x.arg for x in a.args]
            kwo = [x.arg for x in a.kwonlyargs]
            pos_def = [ast.literal_eval(d) for d in a.defaults]
            kw_def = [None if d is None else ast.literal_eval(d) for d in a.kw_defaults]
            return pos, dict(zip(pos[len(pos) - len(pos_def):], pos_def)), kwo, dict(zip(kwo, kw_def))
    raise AssertionError(name)


def _torch_signature(fn):
    sig = inspect.signature(fn)
    pos = [p.name for p in sig.parameters.values() if p.kind == p.POSITIONAL_OR_KEYWORD]
    kwo = [p.name for p in sig.parameters.values() if p.kind == p.KEYWORD_ONLY]
    pos_def = {p.name: p.default for p in sig.parameters.values()
               if p.kind == p.POSITIONAL_OR_KEYWORD and p.default is not p.empty}
    kw_def = {p.name: p.default for p in sig.parameters.values() if p.kind == p.KEYWORD_ONLY}
    return pos, pos_def, kwo, kw_def


@pytest.mark.parametrize("module,name,torch_path", [
    ("flash", "flash_attention", "algx.kernels.flash"),
    ("fused_head", "fused_head", "algx.kernels.fused_head"),
    ("qk_norm", "qk_rms_norm", "algx.kernels.qk_norm"),
])
def test_shim_signatures_match_the_reference(module, name, torch_path):
    """The JAX shims take the reference's arguments (kernels/flash.py:763-772,
    fused_head.py:260, qk_norm.py:62), as the torch front-end does."""
    mod = importlib.import_module(torch_path)
    assert _shim_signature(module, name) == _torch_signature(getattr(mod, name))


def test_front_ends_share_the_variant_module():
    from algx import variants
    from algx.kernels import flash, fused_head
    assert flash.make_variant is variants.make_variant
    assert flash.config_lists is variants.config_lists
    assert fused_head.head_config_lists is variants.head_config_lists
    for f in os.listdir(SHIMS):
        if f in ("flash.py", "fused_head.py", "qk_norm.py"):
            assert "from algx import variants as VA" in open(os.path.join(SHIMS, f)).read()


@pytest.mark.skipif(not HAS_JAX, reason="jaxlib is not installed in this image")
def test_handlers_compile_against_jaxlib():
    import jax.ffi
    subprocess.run(["g++", "-std=c++17", "-fsyntax-only", f"-I{jax.ffi.include_dir()}",
                    f"-I{os.path.join(ROOT, 'include')}", "-I/usr/local/cuda/include", CC], check=True)


@pytest.mark.gpu
@pytest.mark.skipif(not HAS_JAX, reason="jaxlib is not installed in this image")
def test_jax_shims_match_the_torch_front_end():
    """QK norm -> guarded asinh attention and the ce head through JAX, against
    the torch front-end on the same inputs (bf16 bar 2e-2)."""
    import numpy as np
    import torch
    sys.path.insert(0, os.path.join(PKG, "jax_ffi"))
    import build as jbuild
    jbuild.build()
    import jax
    import jax.numpy as jnp
    import algx_jax
    from algx.kernels import flash as TF
    from algx.kernels import qk_norm as TQ
    rng = np.random.default_rng(0)
    q, k, v, do = (rng.standard_normal((1, 2, 256, 64)).astype(np.float32) for _ in range(4))
    gain = (1 + 0.02 * rng.standard_normal(64)).astype(np.float32)

    def jloss(q, k, v, gain):
        qn = algx_jax.qk_rms_norm(q.astype(jnp.bfloat16), gain)
        o = algx_jax.flash_attention(qn, k.astype(jnp.bfloat16), v.astype(jnp.bfloat16), kind="asinh", n=16, c=8.,
                                     range_guard=True)
        return jnp.sum(o.astype(jnp.float32) * do)

    jg = jax.grad(jloss, argnums=(0, 1, 2, 3))(q, k, v, gain)
    tl = [torch.from_numpy(x).cuda().to(torch.bfloat16).requires_grad_(True) for x in (q, k, v)]
    tg = torch.from_numpy(gain).cuda().requires_grad_(True)
    o = TF.flash_attention(TQ.qk_rms_norm(tl[0], tg), tl[1], tl[2], kind="asinh", n=16, c=8., range_guard=True)
    torch.sum(o.float() * torch.from_numpy(do).cuda()).backward()
    for a, b in zip(jg, [t.grad for t in tl] + [tg.grad]):
        a64, b64 = np.asarray(a, np.float64), b.double().cpu().numpy()
        assert np.linalg.norm(a64 - b64) <= 2e-2 * np.linalg.norm(b64)
