"""CPU oracle for the fp32 GEMM path (test infrastructure only; see oracle.py)."""
