"""CPU oracle for the ntilang_b200 hot path — TEST INFRASTRUCTURE ONLY.

Importable by ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline legs,
and only there, as the checker or the timed CPU baseline.  The product path never uses it.

* ``ntl_oracle``  NumPy restatements of each op in the reference's operation order.
* ``rowops``      ctypes loader for the C/OpenMP restatement of the row ops (``rowops.c``).
"""
