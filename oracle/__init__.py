"""CPU oracle of the SPO learner step (test infrastructure only; see spo_oracle)."""
