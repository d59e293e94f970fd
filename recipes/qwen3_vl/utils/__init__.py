"""Recipe-local utilities."""
