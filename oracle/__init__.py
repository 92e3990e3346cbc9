"""CPU oracle for the DS hot path.

Test infrastructure only: ``tests/``, ``__graft_entry__.smoke()`` and the
CPU-baseline leg of ``bench.py`` import it as the checker.  The product
(``ds_b200``) never imports it.
"""
