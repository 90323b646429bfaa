"""ORACLE — test infrastructure only: a CPU restatement of the reference's
behavioural model that tests/, __graft_entry__.smoke() and the cpu_baseline /
reference legs of bench.py compare the engine's results against. The product never imports it."""
