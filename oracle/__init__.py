"""CPU oracle for the parity tests (test infrastructure, never the product)."""
