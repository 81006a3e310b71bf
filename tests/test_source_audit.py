"""Source audit: the algebraic paths compute no exponential or logarithm.

The reference's algebraic model promises arithmetic, comparisons and
reciprocal roots only (model.py:1-8, the primitive audit of
audit_algebraic.py). On this side that holds for the CUDA sources: the tcgen05
attention kernels, the QK norm, the RMS norm and ALU-GLU contain no
transcendental call at all, and every exp/log call that remains in the generic
attention kernels or the head serves the softmax / cross-entropy kind only,
behind that kind's guard.
"""

import os
import re

import pytest

CSRC = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "algebraic-extra_b200", "csrc")
CALL = re.compile(r"\b(?:__)?(?:expf?|exp2f|expm1f|logf?|log2f|log1pf|powf|__expf|__logf)\s*\(|\b(?:ex2|lg2)\.approx")


def _code_lines(name):
    """Source lines with // comments removed (block comments are not used in csrc)."""
    with open(os.path.join(CSRC, name)) as f:
        return [line.split("//", 1)[0] for line in f.read().split("\n")]


def _calls(name):
    return [(i + 1, line) for i, line in enumerate(_code_lines(name)) if CALL.search(line)]


@pytest.mark.parametrize("name", ["attn_tc.cu", "attn_tc.h", "attn_common.cuh", "sm100.cuh", "qknorm.cu",
                                  "vec_io.cuh", "algx_common.cuh"])
def test_no_transcendental_in_algebraic_kernels(name):
    assert _calls(name) == []


def test_model_ops_transcendentals_only_in_the_swiglu_sigmoid():
    lines = _code_lines("model_ops.cu")
    calls = _calls("model_ops.cu")
    assert calls and all("sigmoid_f" in line for _, line in calls), calls
    users = [i + 1 for i, line in enumerate(lines) if "sigmoid_f(" in line and "__device__" not in line]
    text = "\n".join(lines)
    for kernel in ("swiglu_fwd_kernel", "swiglu_bwd_kernel"):
        assert kernel in text
    # every use of the sigmoid lies inside a SwiGLU kernel, none in ALU-GLU or the norms
    starts = {m.start(): m.group(1)
              for m in re.finditer(r"__global__\s+void\s+(?:__launch_bounds__\([^)]*\)\s+)?(\w+)\s*\(", text)}
    assert users
    offsets = [sum(len(l) + 1 for l in lines[:n - 1]) for n in users]
    for off in offsets:
        owner = max((s for s in starts if s < off), default=None)
        assert owner is not None and starts[owner].startswith("swiglu_"), starts.get(owner)


@pytest.mark.parametrize("name,guards", [
    ("attn_generic.cu", ("BR_SOFTMAX",)),
    ("head.cu", ("ALGX_HEAD_CE",)),
])
def test_remaining_transcendentals_serve_the_softmax_kinds(name, guards):
    """Each call site has its kind's guard in the 16 lines up to it; an `else`
    that closes an if-chain over both asinh branches (unshifted, shifted) is the
    softmax branch by elimination."""
    lines = _code_lines(name)
    calls = _calls(name)
    assert calls  # the softmax / ce paths do use exp and log
    for n, line in calls:
        window = "\n".join(lines[max(0, n - 17):n])
        by_guard = any(g in window for g in guards)
        by_elimination = "BR_UNSHIFTED" in window and "BR_SHIFTED" in window and "else" in lines[n - 2] + line
        assert by_guard or by_elimination, f"{name}:{n}: {line.strip()}"
