"""CPU oracle of the MoE / QMoE hot path (test infrastructure only)."""
