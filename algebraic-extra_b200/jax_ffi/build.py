"""Build libalgx_jax.so, the XLA FFI handlers over libalgx (algx_jax_ffi.cc).

Needs jaxlib (for ``jax.ffi.include_dir()``, which holds ``xla/ffi/api/ffi.h``)
and a built ``algx/libalgx.so``. Run ``python jax_ffi/build.py`` from
``algebraic-extra_b200``; the library lands next to libalgx.so, where
``algx_jax`` looks for it.
"""

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
ROOT = os.path.dirname(PKG)
LIBDIR = os.path.join(PKG, "algx")


def build(cxx: str = "g++") -> str:
    try:
        import jax.ffi
    except ImportError as e:  # pragma: no cover - depends on the environment
        raise RuntimeError("building the jax.ffi handlers needs jaxlib (jax.ffi.include_dir())") from e
    out = os.path.join(LIBDIR, "libalgx_jax.so")
    cmd = [cxx, "-O2", "-std=c++17", "-shared", "-fPIC", f"-I{jax.ffi.include_dir()}",
           f"-I{os.path.join(ROOT, 'include')}", "-I/usr/local/cuda/include", os.path.join(HERE, "algx_jax_ffi.cc"),
           f"-L{LIBDIR}", "-lalgx", f"-Wl,-rpath,{LIBDIR}", "-o", out]
    subprocess.run(cmd, check=True)
    return out


if __name__ == "__main__":
    print(build(*sys.argv[1:]))
