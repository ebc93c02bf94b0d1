"""CPU oracle of the H3 step: test infrastructure only (see h3_oracle.py)."""
