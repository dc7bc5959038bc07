"""Test-only CPU oracle for the FxPR hot path (see fxp_oracle.py header)."""
