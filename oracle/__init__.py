"""CPU oracle for the GEMM path. Test infrastructure only: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU baseline, never by the product package."""
