"""CPU oracle for the MoE FFN hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, in NumPy, the reference's NumPy oracles and MLIR
components for ``moe_ffn_block`` / ``mul_mat_id`` / ``swiglu``.  It is the
checker the CUDA path is compared against and the CPU baseline that
``bench.py`` times.  Only ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py`` (its CPU-baseline and ``--impl reference`` legs) may import it;
the product package never does.

Parity pin: ``tests/golden/make_golden.py`` runs the reference's own
``oracles/moe.py`` and ``oracles/activation.py`` on seeded inputs and stores
inputs and outputs as fixtures; ``tests/test_oracle_golden.py`` checks this
restatement against every fixture.
"""
