"""CPU oracle of the quantized DiT-block hot path -- TEST INFRASTRUCTURE ONLY.

A restatement, in numpy/torch on the CPU, of the reference's algorithm for each function on the path
(chronarion/fasth3-gb300, citations are file:line in that project). Only ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU-baseline leg may import it, and only as the checker or the timed CPU baseline: the product path
(``fasth3-gb300_b200/``) never calls it and has no CPU fallback.

Pinning: ``tests/golden/`` holds outputs of the reference's own CUDA kernels (``h3fast.cu`` built from its source for
sm_100a by ``oracle/ref_build/build_ref.py`` and run on a B200 by ``tests/golden/gen_golden.py``); the CPU tests check
this oracle against them. The reference ships no golden vectors of its own.
"""
