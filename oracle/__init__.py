"""CPU oracle (test infrastructure only): restatements of the reference's arithmetic used as the checker by tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline leg. Never imported by the product path."""
