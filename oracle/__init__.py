"""CPU oracles for the CKL hot path.  TEST INFRASTRUCTURE ONLY.

Nothing on the product path imports this package; it exists so the tests, ``smoke()`` and
the CPU-baseline legs of ``bench.py`` can check and time the reference algorithm on the host.
"""
