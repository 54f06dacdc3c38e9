"""CPU oracle (test infrastructure only; see bio_oracle.py)."""
