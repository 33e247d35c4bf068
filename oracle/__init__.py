"""CPU oracle for the paged-KV hot path of mini-inference.

TEST INFRASTRUCTURE ONLY. Nothing in the product package imports this
directory. Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline
leg of ``bench.py`` (its ``cpu_baseline`` measurement and ``--impl reference``)
may import it, and only as the checker or as the timed CPU restatement of
the reference, never as a code path of the product.

Contents:

* :mod:`oracle.block_manager` -- pure-Python restatement of the reference's
  block allocator and prefix cache (``engine/kv_cache.py:377-560``).
* :mod:`oracle.paged_kv` -- numpy restatement of the KV append, write index /
  slot_mapping, paged decode attention and packed (varlen) prefill attention
  (``engine/kv_cache.py:218-301,562-624`` and ``engine/model.py:101-147``).

Parity is pinned: ``tests/test_oracle_golden.py`` checks both modules against
fixtures in ``tests/golden/`` that ``tests/golden/make_golden.py`` produced by
running the reference's own code.
"""
