"""CPU oracle for the beam-decode hot path -- TEST INFRASTRUCTURE ONLY.

This package is a plain Python/numpy restatement of the reference engine
(brian030128/beam_engine) for the path the B200 build replaces: the FIFO page
allocator and paged KV pools, the beam trie with copy-on-write forks, the
cascade and FastTree metadata builders, the attention semantics those
metadata drive (FlashInfer's multi-level cascade, paged append, paged
prefill; the FastTree two-stage kernel), the vanilla beam strategy and a
numpy Llama decoder for end-to-end token parity.

It is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py`` (its ``cpu_baseline`` leg and the
``--impl reference`` arm) may import it.  The product package
``beam_engine_b200`` never imports anything from here and fails loudly when
its CUDA library is missing.

Pinning: the integer parts (allocator order, trie forks, cascade levels,
FastTree vnode metadata) are pinned against fixtures produced by running the
unmodified reference Python in the build container
(``tests/golden/make_golden.py``).  The FastTree attention math is pinned
against the reference's own Triton kernel run under the Triton interpreter.
FlashInfer's CUDA kernels (cascade/prefill/append) cannot run without a GPU
and are not vendored by the reference, so their semantics are restated from
FlashInfer's published Python API; the cascade restatement is cross-checked
against dense attention built from the reference's own ``req_to_token``
tables.  That boundary is "parity pinned by restatement" rather than by a
reference run.
"""
