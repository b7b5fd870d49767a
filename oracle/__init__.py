"""CPU oracle for the GLM path (test infrastructure: the checker, not the product)."""
