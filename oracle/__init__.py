"""ORACLE — test infrastructure only: a CPU restatement of the reference's
behavioural model used as the checker by tests/, __graft_entry__.smoke() and the
cpu_baseline / reference legs of bench.py. The product never imports it."""
