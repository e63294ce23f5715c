"""CPU oracle of the reference's fused decode path.

Test infrastructure only: used by tests/, __graft_entry__.smoke() and the CPU
baseline of bench.py, never by the product package.
"""
