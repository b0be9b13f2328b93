"""CPU oracle (test infrastructure only; see attention_oracle.py)."""
