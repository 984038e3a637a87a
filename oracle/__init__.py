"""Test infrastructure: the CPU oracle for zipfft_b200's correlation path.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
arm may use this package, and only as the checker or the timed CPU baseline --
never as the product path.  See xcorr_oracle.py for the algorithm and the
reference lines each function restates.
"""
