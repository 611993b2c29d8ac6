"""CPU oracle of the enGPT forward path -- test infrastructure, not product code.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
legs import this package.  See ngpt_oracle.py.
"""
