"""Test infrastructure: the CPU checker for the ffwd_b200 CUDA path.

``oracle.forward`` restates the reference CPU forward in numpy; ``oracle.ref``
drives the reference's own CPU code compiled from its sources into
``oracle/_ref``.  Only tests, ``__graft_entry__.smoke()`` and ``bench.py``'s
CPU-baseline leg use this package; the product never imports it.
"""
