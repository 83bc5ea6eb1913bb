"""CPU restatement of the reference algorithms: test infrastructure only (see kata_oracle.py)."""
