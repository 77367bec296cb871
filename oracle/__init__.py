"""Test infrastructure: CPU oracle of the reference algorithm (never on the product path)."""
