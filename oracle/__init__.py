"""CPU oracle for the PageGauge decode path -- TEST INFRASTRUCTURE ONLY.

Nothing in the product (``pagegauge_b200``) imports this package.  It is
used by ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` as the checker the CUDA kernels are compared against.

Pinning: ``oracle/pagegauge_oracle.py`` is validated against
  * golden vectors produced by the reference's own CPU-importable code
    (``quantize_page_gauge``), committed under ``tests/golden/`` together
    with the generating script, and
  * the reference's known-answer lists and formula pins (page tables,
    RoPE expression, Triton scale algebra), restated in ``tests/``.
The reference's append/tail-merge CUDA extension can also be compiled into
``oracle/_ref/`` (``oracle/build_ref.py``) and run on a GPU as a second,
bit-exact checker.
"""
