"""CPU oracle for the AKV cache-operation path: TEST INFRASTRUCTURE ONLY.

Imported by tests/, ``__graft_entry__.smoke()`` and the cpu_baseline leg of
bench.py as the checker.  The product package ``akv_b200`` never imports it.
"""
