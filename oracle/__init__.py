"""CPU oracle for the Q8_0-weight x FP32-activation contraction path.

TEST INFRASTRUCTURE ONLY. This package restates, in NumPy, the reference
(mgostIH/parakeet_cuda) algorithm for the hot path so that the CUDA library
can be checked against it:

* ``oracle.q8``  - Q8_0 block decode, float64 GEMM/GEMV goldens, fused
  epilogue math and a TF32 rounding model of the tensor-core operands.
* ``oracle.tdt`` - the TDT prediction/joint network and the greedy token loop.
* ``oracle.cpu_path`` - the reference's NumPy CPU linear (decode to FP32 then
  ``x @ W.T``), used only as the timed CPU baseline in ``bench.py``.

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` leg of ``bench.py`` may import it, and only as the checker
or the reported CPU baseline. The product (``parakeet_cuda_b200``) never calls
into it and has no CPU fallback.

Parity is pinned: ``tests/test_oracle_golden.py`` checks this oracle against
golden vectors produced by running the reference's own code
(``tests/golden/make_golden.py``).
"""
