"""CPU oracle of Sarbon's temporal block-sparse engine -- test infrastructure only.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may
import this package; the product path (``sarbon_b200``) never does.
"""
