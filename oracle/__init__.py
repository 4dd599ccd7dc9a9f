"""CPU oracle: test infrastructure only (see sampling_oracle.py)."""
