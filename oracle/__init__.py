"""CPU oracle of the quantized-linear path -- test infrastructure only (see qpu_oracle.py)."""
