"""CPU oracle for the attention forward (test infrastructure; never on the product path)."""
