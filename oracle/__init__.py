"""CPU oracle for the parity tests and the CPU baseline (test infrastructure)."""
