"""TEST INFRASTRUCTURE ONLY: CPU checkers for blackflash_b200 (never on the product path)."""
