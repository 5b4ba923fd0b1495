"""CPU oracle for the gated delta-rule path.  TEST INFRASTRUCTURE ONLY: imported
by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg as the
checker; the product path never calls it."""
