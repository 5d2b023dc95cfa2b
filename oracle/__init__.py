"""CPU oracle for the H3 Ulysses attention path (test infrastructure only; see h3_oracle)."""
