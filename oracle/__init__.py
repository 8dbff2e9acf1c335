"""CPU oracle for the W4A8 ConvRot qlinear (test infrastructure only; see qlinear_oracle.py)."""
