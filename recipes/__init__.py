"""Training recipes (engines + configs) built on mvp_engine."""
