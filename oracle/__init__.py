"""Test-only CPU oracle for the H3 DiT-block hot path (see h3_oracle.py)."""
