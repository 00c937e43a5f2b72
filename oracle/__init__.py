"""CPU oracle for paged split-K GQA decode attention. TEST INFRASTRUCTURE ONLY.

Nothing in the product package imports this directory.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm use
it, and only as the checker or as the timed CPU baseline, never as the product.

Contents
--------
``paged_oracle``   FP64 NumPy restatement of the reference's oracle
                   (src/paged_decode/oracle.py:30-117 of ensigncode/paged-decode-lab).
``c_oracle``       ctypes front end of ``paged_oracle.c``: the same FP64 dense
                   attention in C, threaded over (sequence, head) rows, used for
                   large parity cases and as the timed CPU baseline.

Parity is pinned: ``tests/golden/*.npz`` were produced by importing the
reference's own Python oracle (``tests/golden/make_golden.py``) and
``tests/test_oracle_golden.py`` checks both restatements against them.
"""
