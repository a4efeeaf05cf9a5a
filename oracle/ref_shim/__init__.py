"""Builds the reference's BaseLM shaders as a CPU library (test infrastructure only; see build_ref.py)."""
