"""serving."""
