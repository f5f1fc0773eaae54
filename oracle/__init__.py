"""CPU oracle for the streaming denoising hot path — TEST INFRASTRUCTURE ONLY.

This package restates, in numpy / PyTorch-on-CPU, the reference's algorithm
for each function on the hot path, citing the reference file:line it follows.
It is the checker: only ``tests/``, ``__graft_entry__.smoke()`` and the CPU
baseline legs of ``bench.py`` may import it.  The product (``reflex_b200``)
never imports it and has no CPU fallback.

Parity pins: the restatement is checked against golden vectors produced by
running the reference's own classes (``tests/golden/make_golden.py``) — the
uint8 KV quantizer bit-exactly, attention / layers / denoise chunk to fp32
rounding.  The int8 symmetric scheme and the scale/shift/gate adaRMS variant
have no reference implementation: the first is pinned by hand-derived
known-answer vectors from its formula, the second is "parity unpinned".
"""
