"""CPU oracle for the paged-KV path (test infrastructure only; see oracle.py)."""
