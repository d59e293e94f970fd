"""Recipe-local helpers (none needed beyond the shared kits)."""
