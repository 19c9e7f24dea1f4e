"""CPU oracle of the PESQ pipeline (test infrastructure only, see pesq_oracle)."""
