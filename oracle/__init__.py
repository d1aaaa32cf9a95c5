"""CPU oracle (test infrastructure only; see oracle/vx_oracle.h)."""
