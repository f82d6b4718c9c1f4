"""CPU oracle for the cvattn engine -- test infrastructure only (see oracle.py)."""
