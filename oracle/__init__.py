"""CPU checkers for the CUDA path. TEST INFRASTRUCTURE ONLY: nothing in the product imports
this package; tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use it as the
checker, never as the thing measured or shipped.

  exact.py  exact big-integer restatement of the reference's ground truth (small cases)
  ref.py    driver for the reference's own C++ certified kernel, compiled into _ref/ by the
            Makefile here from the reference's source file; flagged rows go to exact.py
"""
