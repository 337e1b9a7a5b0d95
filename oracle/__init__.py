"""CPU oracle for the mlxz KV-cache hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, what the reference (metazen11/mlxz) computes
on its KV-cache path, each function citing the reference file:line it follows.
It is the checker: only ``tests/``, ``__graft_entry__.smoke()`` and the CPU
baseline legs of ``bench.py`` may import it.  The product (``mlxz_b200``)
never imports or calls it, and has no CPU fallback.

Pinning.  ``tests/golden/`` holds vectors produced by running the reference's
own ``paged_kv.py`` / ``attention.py`` / ``block_manager.py`` /
``prefix_cache`` sources under a torch-CPU stand-in for ``mlx.core``
(``tests/golden/make_golden.py``); ``tests/test_oracle_golden.py`` checks this
oracle against them.  Parity is pinned for append, gather, attention
(softmax(q.K^T*s).V with the h // G GQA mapping; MLX's own SDPA kernel is not
runnable here, so its rounding is unpinned), block allocation and prefix-cache
policy.  Affine 4/8-bit quantisation follows MLX's published definition; no
reference test or runnable MLX pins its rounding ("parity unpinned" for the
quantised packing).
"""
