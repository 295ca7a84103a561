"""CPU oracle for the omniASR-LLM decoder-attention hot path -- TEST INFRASTRUCTURE ONLY.

A plain restatement of the reference's algorithms (Wataru-Nakata/omniasr-trt; each function cites the reference
file:line it follows), used as the checker of the CUDA kernels. Only ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py`` (its CPU baseline and ``--impl reference`` arm) may import it; the product path
(``omniasr_b200``) never does and has no CPU fallback.

* :mod:`oracle.bf16`      -- bfloat16 <-> float32 conversions in numpy (round-to-nearest-even, bit-exact)
* :mod:`oracle.rope`      -- RoPE + KV-cache append, bit-exact (numpy)
* :mod:`oracle.gather`    -- beam reorder gather, byte-exact (numpy)
* :mod:`oracle.attention` -- decode / draft / beam / prefill attention (torch, fp64 by default)
* :mod:`oracle.splits`    -- the reference's key-split rule

Pinning: ``tests/golden/`` holds vectors produced by running the reference's own code in the build container
(``tests/golden/make_golden.py``); ``tests/test_oracle.py`` checks this oracle against every one of them.
"""
