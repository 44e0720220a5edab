"""GEMM calibration: the measured matmul rates the cost model prices work at."""
