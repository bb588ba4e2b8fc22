"""CPU oracle for the mingru scan family (test infrastructure only; see oracle.py)."""
