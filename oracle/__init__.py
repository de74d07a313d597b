"""CPU oracle for the LLMY looped hybrid block hot path — TEST INFRASTRUCTURE.

These modules restate, in numpy (fp64 unless noted), the reference
algorithms of StillPillWill/Hybrid_LLM that the CUDA kernels replace.  Each
function cites the reference file:line it follows.  The restatements are
pinned against golden vectors produced by running the reference's own PyTorch
code (``tests/golden/make_golden.py``).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may import this package, and only as a checker or as the timed CPU
baseline.  The product path (``hybrid_llm_b200``) never imports it.
"""
