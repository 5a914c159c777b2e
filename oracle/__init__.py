"""CPU checker for the CUDA path (test infrastructure; never imported by the product)."""
