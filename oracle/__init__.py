"""CPU oracle of the W8A8 path (test infrastructure only; see w8a8.py)."""
