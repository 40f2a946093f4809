"""CPU oracle for the Lngram v2 route n-gram memory path (TEST INFRASTRUCTURE ONLY).

This package restates, in numpy (and plain C for the integer addressing), the
reference algorithm of MorbiusPlexus/lngram-decode for the memory lookup,
the memory readout, the draft head, tree addressing and the per-token drafter.
Every function cites the reference file:line it follows.

It is the checker, never the product: only ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py``'s CPU-baseline leg may import it.  The package
``lngram-decode_b200`` never imports it and has no CPU fallback.

Pinning: ``tests/test_oracle_reference_pins.py`` checks this oracle against
the reference's own stored golden logits (``tests/data/wave1_reference.npz``,
with this oracle substituted for the memory layer) and against the reference
modules run in this container; ``tests/golden/make_golden.py`` writes the
fixtures that the CPU and GPU tests replay without the reference present.
"""
