"""CPU oracle for the contraction hot path (test infrastructure only)."""
