"""CPU oracle of the quantized Titan-block forward -- TEST INFRASTRUCTURE ONLY.

Imported only by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
leg, as the checker or the timed CPU baseline; never by the product path.
"""
