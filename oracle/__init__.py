"""CPU oracle of the fused layer ops — TEST INFRASTRUCTURE ONLY.

Used by tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg
as the checker; the product package ``anima_flat_b200`` never imports it.

``canonical``: oracle.c, a C restatement of the reference's formulas with the
canonical reduction order the CUDA kernels follow (bit-exact target).
``formulation``: the reference's unfused PyTorch-eager fp32 composition
(tolerance target, and the timed CPU baseline).

Parity of the canonical oracle is pinned against golden vectors that
tests/golden/gen_golden.py produced by running the reference's own Triton
kernels under TRITON_INTERPRET=1 (mode=INTERP reproduces that interpreter's
casts and numpy reduction order).
"""
