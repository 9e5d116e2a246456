"""The parity oracle: a CPU restatement of the reference's decoder-attention path -- TEST INFRASTRUCTURE ONLY.

* :mod:`oracle.attn`  -- the attention ops of the reference's ``src/whisper_trt/attn_plugin.py`` (numpy, float32)
* :mod:`oracle.slots` -- the slot-table / beam bookkeeping of ``search.py`` and ``beam_kernels.py`` (numpy, ints)

Pinned: ``tests/golden/make_golden.py`` runs the reference itself (imported from its source tree, on CPU) on the
seeded cases of ``tests/golden/cases.py`` and stores its outputs under ``tests/golden/``; ``tests/test_oracle_golden.py``
checks this oracle against them. Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs (the
``cpu_baseline`` sample and ``--impl reference``) may import this package: it is the checker, never the product,
and the product path has no CPU fallback.
"""
