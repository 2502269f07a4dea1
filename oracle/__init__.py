"""CPU oracle of the reference attention path -- TEST INFRASTRUCTURE ONLY.

Imported by tests/, __graft_entry__.smoke() and the CPU-baseline leg of
bench.py as the checker; never by the product package (minisgl_b200).
"""
