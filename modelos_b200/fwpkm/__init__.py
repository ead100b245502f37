"""Fast-weight product-key memory (the reference's ``fwpkm`` package)."""
