"""CPU/FP32 oracle for the HGEMM hot path. Test infrastructure only: imported
by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg, never by
the llm_hgemm product code."""
