"""CPU oracle (test infrastructure only): see ``pkm_oracle``.

Only tests, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline legs may
import this package; the product package never does.
"""
