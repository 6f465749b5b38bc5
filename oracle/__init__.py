"""CPU oracle for the FlashHead decode-step head: TEST INFRASTRUCTURE ONLY.

Imported only by tests/, __graft_entry__.smoke() and bench.py's CPU legs, as
the checker or the timed CPU baseline; never by the flash_head package.
"""
