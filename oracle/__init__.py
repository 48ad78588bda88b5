"""Parity oracle for the CUDA backend (test infrastructure only; see gcdr_oracle.py)."""
