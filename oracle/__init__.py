"""CPU oracle for the SDPA forward — test infrastructure only (see oracle.py)."""
