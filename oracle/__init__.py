"""CPU oracle of the MoE hot path: test infrastructure only (see moe_oracle.py)."""
