"""CPU oracle of the MoE hot path.  TEST INFRASTRUCTURE ONLY: imported by tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline arm, never by easyinfra_b200."""
