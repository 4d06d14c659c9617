"""CPU oracle of the BA linearization path (test infrastructure; never imported by the product)."""
