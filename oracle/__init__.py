"""Test infrastructure only: the CPU oracle for the attention-backward path.

Nothing in the product (the ``attn_bwd_b200`` package and its CUDA library)
imports this package; only ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU-baseline / reference arm use it, as the checker or as the
timed CPU reference.
"""
