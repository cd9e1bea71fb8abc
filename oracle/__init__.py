"""CPU oracle for the HSTU jagged attention path.  TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline / reference
legs of ``bench.py`` may import this package; the product package
``recir_b200`` never does.
"""
