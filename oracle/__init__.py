"""CPU oracle of the token loop -- test infrastructure only (see spm_oracle.h)."""
