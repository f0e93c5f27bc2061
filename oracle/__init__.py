"""CPU checkers for the attention engine (test infrastructure only)."""
