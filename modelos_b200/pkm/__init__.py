"""Slow-weight product-key memory (the reference's ``pkm`` package)."""
