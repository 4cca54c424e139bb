"""CPU oracle for the attention hot path — TEST INFRASTRUCTURE ONLY.

Imported only by tests/, __graft_entry__.smoke() and bench.py's CPU baseline
leg.  The product package never imports it.
"""
