"""CPU oracle for the MoE-expert hot path (test infrastructure only).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg import
this package; the product under ``minirun-app_b200/`` never does.
"""
