"""CPU oracle for the routed-expert hot path (test infrastructure only)."""
