"""Parity oracle for the FG-CPAB hot path (test infrastructure only)."""
