"""CPU oracle of the FP8 MoE hot path. TEST INFRASTRUCTURE: imported only by
tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg, as the
checker — never by the product package."""
