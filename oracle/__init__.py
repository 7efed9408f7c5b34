"""Test-only CPU oracle (fp32 restatement of the reference's torch path).

Imported only by tests/, __graft_entry__.smoke() and bench.py's CPU baseline
legs; never by the mega_trading_b200 product package.
"""
