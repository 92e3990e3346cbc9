"""CPU oracle for the DS hot path.

Test infrastructure only: ``tests/``, ``__graft_entry__.smoke()`` and the
CPU-baseline leg of ``bench.py`` import it to check results against.  The
product (``ds_b200``) never imports it.
"""
