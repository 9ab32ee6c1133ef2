"""CPU oracle for the speculative path (test infrastructure only; never imported by the product)."""
