"""CPU oracle for the CORE compression step (test infrastructure only; see core_oracle)."""
