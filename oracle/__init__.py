"""CPU oracle of the l0llm decoder hot path: test infrastructure only (see l0b_oracle.h)."""
