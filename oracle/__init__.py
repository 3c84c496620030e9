"""CPU oracle for the needle attention hot path (test infrastructure only)."""
