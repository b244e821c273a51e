"""CPU oracle for parity tests — TEST INFRASTRUCTURE, never the product path.

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import this package. The shipped
backend (``mdlc_b200``) never imports it and has no CPU fallback.

* :mod:`oracle.reference` restates the reference NumPy executor
  (``mdlc/runtime/reference.py`` + ``mdlc/runtime/ops.py``) and extends it with
  the ops the reference lacks (``Erf``, ``ReduceMean``). Pinned against
  fixtures produced by importing the reference itself
  (``tests/golden/make_golden.py``).
* :mod:`oracle.quant` is the INT8 restatement (calibration, per-channel weight
  quantisation, int32 accumulation, fp32 / fixed-point requantisation). The
  reference has no quantised ops, so its parity is defined by this restatement
  ("parity unpinned by the reference" for INT8).
"""
