"""CPU oracle of the SwiGLU-MLP recompute path (test infrastructure only)."""
