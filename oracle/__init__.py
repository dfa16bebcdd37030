"""CPU oracle of the attention-share audit and block-table view path -- TEST INFRASTRUCTURE ONLY.

This package restates, in plain numpy, the reference algorithm of every function on the hot path,
each citing the reference file:line it follows. It is the checker the parity tests compare the
sm_100a kernels against, and the CPU baseline ``bench.py`` times. Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py`` (its CPU-baseline leg, ``--impl reference``, and the
parity check it runs after its timed regions) may import it; the product (``ekv``) never does.

Parity of the oracle itself is pinned against golden vectors produced by running the reference's
own code (``tests/golden/make_golden.py``: the Triton audit kernel under ``TRITON_INTERPRET=1``, the
reference normalisation, allocation and compaction) and against the known answers of the reference's
own unit tests.
"""
