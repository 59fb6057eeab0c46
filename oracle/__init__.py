"""CPU checkers for the FastGS rasterizer (test infrastructure only)."""
