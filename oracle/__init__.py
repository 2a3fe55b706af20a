"""CPU oracle for the MaskAhead select + attend hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU, the algorithm of the reference implementation
(brain-lab-research/MaskAhead, ``src/maskahead``) for the per-block hot path:
prefix-softmax scoring, value-aware rescoring, top-k read-set selection, lookahead
retention survivors, dense step-0 attention and the sparse sub-step attention, plus
the packed uint4 cache formats that define the inputs.

Every function cites the reference file:line it follows. Floating-point work runs in
torch fp32 on the CPU (the reference's own CPU path is torch fp32); integer and byte
work (packing, order keys, top-k with an explicit tie rule) is numpy.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may
import this package, and only as the checker or as the timed CPU baseline. The
product package ``maskahead_b200`` never imports it and has no CPU fallback.

Parity pinning: ``tests/golden/make_golden.py`` imports the reference package (in
the build container, where it is mounted) and records its outputs on seeded inputs
into ``tests/golden/*.npz``; ``tests/test_oracle_golden.py`` checks this oracle
against those recorded outputs.
"""

from .ref_math import *  # noqa: F401,F403
