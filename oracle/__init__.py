"""CPU oracle of the attention forward path — test infrastructure only (see attention_oracle)."""
