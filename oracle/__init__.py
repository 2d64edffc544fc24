"""Test infrastructure: the CPU oracle (see oracle.py).  Never imported by
the product package."""
