"""CPU oracle for AceFlow's retention path (test infrastructure only).

``retention_ref`` restates the reference in numpy; ``cpu_ref`` wraps the C
restatement of the Rust SIMD path.  Only ``tests/``, ``__graft_entry__.smoke``
and ``bench.py``'s CPU-baseline leg may import this package.
"""
