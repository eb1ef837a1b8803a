"""CPU oracle for the MedIT One decode path (test infrastructure only).

Nothing in the product package imports this package. Only ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` use it,
and only as the checker / the timed CPU reference.
"""
