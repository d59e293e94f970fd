"""Data for this recipe comes from ``MLLMDataKit`` (lance / json / parquet / synthetic sources)."""
