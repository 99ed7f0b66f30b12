"""CPU oracle -- test infrastructure only (see afa_oracle.py). Imported by tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline leg, never by the product."""
