"""Drop-in replacements for the reference's ``src/kernels`` op modules.

``anima_flat_b200.kernels.adaln``, ``.fp8`` and ``.rope`` expose the public
functions of ``src/kernels/adaln.py``, ``fp8.py`` (activation quantisation)
and ``rope.py`` under the same names and signatures, backed by the sm_100a
C-ABI library.
"""
