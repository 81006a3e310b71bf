"""Drop-in counterparts of the reference's ``algebraic.kernels`` package."""
