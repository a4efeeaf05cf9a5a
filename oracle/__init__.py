"""CPU oracle for the BaseLM decode step (test infrastructure only; see oracle.py)."""
