"""CPU oracle of the StrideWeave hot path (test infrastructure only)."""
