"""CPU oracle -- TEST INFRASTRUCTURE ONLY.

A plain-PyTorch (CPU, fp32/fp64) restatement of the reference's eager
forward passes, used to check the B200 kernels.  Nothing in the product
(``torch-helion_b200/``) imports this package; only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg do, and
only as the checker / the timed CPU baseline, never as the computation that
is measured or shipped.

Pinning: ``tests/test_oracle.py`` checks every function here against golden
vectors produced by the reference's own code (``models/llama_block.py``,
``models/mamba.py`` imported from the reference checkout) by
``tests/golden/make_golden.py``, and against the reference's known-answer
identities (tests/test_mamba.py:27-74 of the reference).

Modules
  models    -- Llama block and Mamba-2 backbone forwards (functional)
  ssd       -- SSD scan: direct recurrence, chunked form, quadratic form
  interpret -- CPU interpreter of a B200 OpIR Program (partition checks)
"""
