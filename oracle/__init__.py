"""TEST INFRASTRUCTURE ONLY: the CPU oracle of the MoE path (see moe_ref.py).

Imported by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg
as a checker; never by the product package.
"""
