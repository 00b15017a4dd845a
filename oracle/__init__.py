"""CPU oracle of the DeLS draft-scoring path — test infrastructure only.

Imported by ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` as the checker / reference timing; never by the product package."""
