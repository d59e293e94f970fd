"""General utilities: registry, logging, metrics, training helpers, checkpointing."""
