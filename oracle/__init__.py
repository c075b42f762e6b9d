"""CPU oracle for futon parity (test infrastructure only)."""
